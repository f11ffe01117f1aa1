"""The oracle pinned to tgc: golden outputs of tgc's interpreter and summation/quantise code,
and tgc's own known-answer assertions (tests/test_summation.py:45,51,119 and
tests/test_quantize.py:95-110 in tgc's tree).
"""

from __future__ import annotations

import hashlib
import json
import math
import os

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import bracketing, interp
from oracle import quantize as oq
from tgcb import ir, serialize, workloads


def sha(t) -> str:
    a = t.numpy() if isinstance(t, torch.Tensor) else t
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_graph(name):
    with open(os.path.join(GOLDEN, "graphs", f"{name}.tgc")) as f:
        return serialize.loads(f.read())


@pytest.fixture(scope="module")
def summ():
    with open(os.path.join(GOLDEN, "summation.json")) as f:
        return json.load(f)


def test_cone_interpreter_matches_tgc():
    gold = np.load(os.path.join(GOLDEN, "cone.npz"))
    feeds = workloads.cone_inputs()
    assert sha(feeds["x"]) == bytes(gold["x_sha"]).decode()
    out = interp.run(workloads.cone_graph(ir.Builder), feeds)
    for o, key in zip(out, ("row_sum", "row_max", "row_sum_tx"), strict=True):
        np.testing.assert_allclose(o.numpy(), gold[key], rtol=2e-6, atol=0)


def test_fixture_graphs_match_tgc():
    gold = np.load(os.path.join(GOLDEN, "fixtures.npz"))
    for name in ("softmax_graph", "layernorm_graph", "diamond_graph", "branching_graph", "mlp_graph"):
        g = load_graph(f"fixture_{name}")
        feeds = {v.name: torch.from_numpy(gold[f"{name}/in/{v.name}"]) for v in g.inputs}
        out = interp.run(g, feeds)
        for i, o in enumerate(out):
            np.testing.assert_allclose(o.numpy(), gold[f"{name}/out/{i}"], rtol=1e-5, atol=1e-6)
        # tgc's generated-Python path restated gives the interpreter's numbers too
        prog = interp.generated_python_program(g)
        for a, b in zip(prog(feeds), out, strict=True):
            assert torch.equal(a, b)


def test_mlp_interpreter_matches_tgc_small():
    gold = np.load(os.path.join(GOLDEN, "mlp.npz"))
    y = interp.run(workloads.mlp_graph(ir.Builder, rows=64), workloads.mlp_inputs(rows=64))[0]
    np.testing.assert_allclose(y.numpy(), gold["y64"], rtol=1e-4, atol=1e-5)


def test_random_feeds_restated():
    g = load_graph("fixture_softmax_graph")
    gold = np.load(os.path.join(GOLDEN, "fixtures.npz"))
    feeds = interp.random_feeds(g, seed=0, positive=True)
    assert np.array_equal(feeds["x"].numpy(), gold["softmax_graph/in/x"])


def test_summation_known_answers(summ):
    k = summ["known"]
    assert k["mixed_4096_sequential"] == 1e9  # tgc tests/test_summation.py:119
    assert k["exact_0.1_0.2_0.3"] == 0.6000000163912773  # tgc tests/test_summation.py:51
    assert bracketing.sequential(np.full(4, 2.5, dtype=np.float32)) == 10.0  # test_summation.py:45
    assert bracketing.pairwise(np.full(4, 2.5, dtype=np.float32)) == 10.0
    assert k["best_split"]["ratio"] > 80


def test_summation_orders_bit_exact(summ):
    gens = {
        "uniform": lambda c, s: np.asarray(np.random.default_rng(s).uniform(0.5, 1.5, size=c), dtype=np.float32),
        "mixed": lambda c, s: np.asarray([1e9, *np.random.default_rng(s).uniform(0.5, 1.5, size=c - 1)], dtype=np.float32),
        "alternating": lambda c, s: np.asarray(np.random.default_rng(s).normal(0.0, 1.0, size=c), dtype=np.float32),
    }
    for vec in summ["vectors"]:
        v = gens[vec["kind"]](vec["count"], vec["seed"])
        assert bracketing.sequential(v) == vec["sequential"]
        assert bracketing.pairwise(v) == vec["pairwise"]
        assert bracketing.pairwise(v, block=3) == vec["pairwise_block_3"]
        if vec["partitioned_64"] is not None:
            assert bracketing.partitioned(v, 64) == vec["partitioned_64"]
        assert math.fsum(v.astype(np.float64).tolist()) == vec["exact"]


@pytest.mark.slow
def test_long_sum_restatement_matches_tgc(summ):
    ls = summ["longsum"]
    v, idx = workloads.longsum_input()
    assert idx == ls["leader_index"]
    assert sha(v) == ls["x_sha"]
    assert bracketing.pairwise(v.numpy()) == ls["pairwise"]
    assert bracketing.sequential(v.numpy()) == ls["sequential"]


def test_quantiser_restatement_bit_exact():
    gold = np.load(os.path.join(GOLDEN, "quantize.npz"))
    for name in ("randn", "weights_t", "edge"):
        x = gold[f"{name}/x"]
        q, s = oq.quantise_rows(x)
        assert np.array_equal(q.astype(np.float32), gold[f"{name}/q"])
        assert np.array_equal(s, gold[f"{name}/scale"].astype(np.float32))
        assert q.min() >= -128 and q.max() <= 127  # tgc tests/test_quantize.py:95-110
        err = np.abs(oq.dequantise_rows(q, s) - x)
        assert np.all(err <= s[:, None] / 2 * (1 + 1e-6))


@pytest.mark.slow
def test_int8_workload_restatement_bit_exact():
    with open(os.path.join(GOLDEN, "int8.json")) as f:
        meta = json.load(f)
    gold = np.load(os.path.join(GOLDEN, "int8.npz"))
    ins = workloads.int8_inputs()
    assert sha(ins["a"]) == meta["a_sha"]
    qa, sa = oq.quantise_rows(ins["a"].numpy())
    qwt, sw = oq.quantise_rows(ins["w"].T.contiguous().numpy())
    assert sha(qa) == meta["qa_sha"] and sha(qwt) == meta["qwt_sha"]
    assert np.array_equal(sa, gold["sa"].reshape(-1)) and np.array_equal(sw, gold["sw"].reshape(-1))
    rows = gold["rows"]
    acc = oq.int_matmul(qa[rows], qwt.T)
    assert np.array_equal(acc, gold["acc_rows"])
    y = (acc.astype(np.float32) * sa[rows, None]).astype(np.float32) * sw[None, :]
    assert np.array_equal(y.astype(np.float32), gold["y_rows"])


def test_gradient_graph_interpreter_matches_tgc():
    gold = np.load(os.path.join(GOLDEN, "train.npz"))
    g = load_graph("train_grad_small")
    feeds = {v.name: torch.from_numpy(gold[f"in/{v.name}"]) for v in g.inputs}
    out = interp.run(g, feeds)
    for i, o in enumerate(out):
        np.testing.assert_allclose(o.numpy(), gold[f"grad_opt/{i}"], rtol=1e-4, atol=1e-7)


def test_row_tree_restatement():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 100)).astype(np.float32)
    for T in (32, 64):
        got = bracketing.row_tree(x, T)
        for r in range(3):
            lanes = []
            for t in range(T):
                acc = np.float32(0)
                for c in range(t, 100, T):
                    acc = np.float32(acc + x[r, c])
                lanes.append(acc)
            while len(lanes) > 1:
                lanes = [np.float32(lanes[i] + lanes[i + 1]) for i in range(0, len(lanes), 2)]
            assert got[r] == lanes[0]
    assert np.array_equal(bracketing.row_tree(x, 32, "max"), x.max(axis=1))
