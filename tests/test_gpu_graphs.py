"""Compiled graphs on the B200 against tgc's interpreter (golden fixtures) and the oracle.

Tolerances: graphs without GEMMs use CUDA's own expf/tanhf/sqrtf (within a few ulp of torch
CPU's) and the declared reduction bracketing, and must agree to rtol 1e-5; reductions over
exactly-representable summands must match the oracle's restatement of the bracketing bit
for bit. Graphs with float32 GEMMs run them on TF32 tensor cores (10-bit mantissa inputs,
fp32 accumulation) and must agree within 5e-3 of the largest output magnitude. int8/int32
work is bit-exact.
"""

from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import bracketing, interp
from oracle import quantize as oq
from tgcb import ir, serialize, workloads
from tgcb.codegen import row_threads
from tgcb.errors import ConfigError
from tgcb.runtime import compile_graph

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3
F32_RTOL = 1e-5


def load_graph(name):
    with open(os.path.join(GOLDEN, "graphs", f"{name}.tgc")) as f:
        return serialize.loads(f.read())


def on_gpu(feeds):
    return {k: v.cuda() for k, v in feeds.items()}


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def run(graph, feeds):
    c = compile_graph(graph)
    out = c(on_gpu(feeds))
    torch.cuda.synchronize()
    c.check_status()
    return c, [o.cpu() for o in out]


def test_cone_full_size_matches_tgc(cuda):
    gold = np.load(os.path.join(GOLDEN, "cone.npz"))
    _, out = run(workloads.cone_graph(ir.Builder), workloads.cone_inputs())
    for o, key in zip(out, ("row_sum", "row_max", "row_sum_tx"), strict=True):
        np.testing.assert_allclose(o.numpy(), gold[key], rtol=F32_RTOL, atol=0)


@pytest.mark.parametrize("rows,cols", [(4096, 1024), (33, 70), (7, 3000), (5, 9000), (1, 1)])
def test_row_reductions_bit_exact_to_declared_bracketing(cuda, rows, cols):
    """sum(x), max(x), sum(x*x), mean(x) per row: summands are exact, so only the order matters."""
    b = ir.Builder()
    x = b.input([rows, cols], name="x")
    g = b.finish(b.sum(x, [1]), b.max(x, [1]), b.sum(b.mul(x, x), [1]), b.mean(x, [1], keepdims=True))
    xv = torch.randn(rows, cols, generator=torch.Generator().manual_seed(rows * 7 + cols))
    _, (s, m, ss, mean) = run(g, {"x": xv})
    T = row_threads(cols, rows)
    xn = xv.numpy()
    assert np.array_equal(s.numpy(), bracketing.row_tree(xn, T))
    assert np.array_equal(m.numpy(), bracketing.row_tree(xn, T, "max"))
    assert np.array_equal(ss.numpy(), bracketing.row_tree(xn * xn, T))
    assert np.array_equal(mean.numpy().reshape(-1), (bracketing.row_tree(xn, T) / np.float32(cols)).astype(np.float32))
    ref = interp.run(g, {"x": xv})
    for o, r in zip((s, m, ss, mean), ref, strict=True):
        assert rel_err(o, r) < 1e-5


@pytest.mark.parametrize("name", ["softmax_graph", "layernorm_graph", "diamond_graph", "branching_graph"])
def test_tgc_fixtures_match_tgc(cuda, name):
    gold = np.load(os.path.join(GOLDEN, "fixtures.npz"))
    g = load_graph(f"fixture_{name}")
    feeds = {v.name: torch.from_numpy(gold[f"{name}/in/{v.name}"]) for v in g.inputs}
    _, out = run(g, feeds)
    for i, o in enumerate(out):
        np.testing.assert_allclose(o.numpy(), gold[f"{name}/out/{i}"], rtol=F32_RTOL, atol=1e-6)


def test_tgc_mlp_fixture_within_tf32(cuda):
    gold = np.load(os.path.join(GOLDEN, "fixtures.npz"))
    g = load_graph("fixture_mlp_graph")
    feeds = {v.name: torch.from_numpy(gold[f"mlp_graph/in/{v.name}"]) for v in g.inputs}
    _, out = run(g, feeds)
    assert rel_err(out[0], torch.from_numpy(gold["mlp_graph/out/0"])) < TF32_TOL


def test_arena_reuse_across_seeds(cuda):
    """tgc's run_many (executor.py:179-193): compile once, reuse one arena, check every seed."""
    g = load_graph("fixture_layernorm_graph")
    c = compile_graph(g)
    arena = c.new_arena()
    for seed in range(6):
        feeds = interp.random_feeds(g, seed=seed, positive=True)
        out = c.function(arena, on_gpu(feeds))
        torch.cuda.synchronize()
        assert rel_err(out[0], interp.run(g, feeds)[0]) < F32_RTOL


def test_mlp_block_full_size_matches_tgc(cuda):
    """Every one of the 8192 output rows against the oracle's interpreter run on this host
    (pinned to tgc's own golden rows and row sums, checked here too), within the TF32
    tolerance of the largest output; and each row within it of its own largest entry."""
    gold = np.load(os.path.join(GOLDEN, "mlp.npz"))
    feeds = workloads.mlp_inputs()
    assert sha(feeds["x"]) == bytes(gold["x_sha"]).decode()
    g = workloads.mlp_graph(ir.Builder)
    _, (y,) = run(g, feeds)
    ref = interp.run(g, feeds)[0]
    rows = gold["rows"]
    np.testing.assert_allclose(ref[rows].numpy(), gold["y_rows"], rtol=1e-4, atol=1e-5)  # the oracle is tgc's
    assert rel_err(y, ref) < TF32_TOL
    per_row = ((y.double() - ref.double()).abs().amax(1) / ref.double().abs().amax(1)).max()
    assert float(per_row) < TF32_TOL
    assert rel_err(y[rows], torch.from_numpy(gold["y_rows"])) < TF32_TOL
    sums = y.double().sum(dim=1).numpy()
    scale = np.abs(gold["y_rows"]).max() * 1024
    assert np.abs(sums - gold["y_row_sums"]).max() / scale < TF32_TOL


def test_mlp_block_small_matches_tgc(cuda):
    gold = np.load(os.path.join(GOLDEN, "mlp.npz"))
    _, (y,) = run(workloads.mlp_graph(ir.Builder, rows=64), workloads.mlp_inputs(rows=64))
    assert rel_err(y, torch.from_numpy(gold["y64"])) < TF32_TOL


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("kind", ["f32", "i8"])
def test_gemm_layouts(cuda, ta, tb, kind):
    """Every operand major for both tensor-core kinds, with ragged M, N and K tiles."""
    M, N, K = 200, 300, 160 if kind == "f32" else 256
    b = ir.Builder()
    ash, bsh = ([K, M] if ta else [M, K]), ([N, K] if tb else [K, N])
    dt = ir.FLOAT32 if kind == "f32" else ir.INT8
    a = b.input(ash, dt, name="a")
    w = b.input(bsh, dt, name="b")
    av, wv = (a, w) if kind == "f32" else (b.cast(a, ir.INT32), b.cast(w, ir.INT32))
    if ta:
        av = b.transpose(av, [1, 0])
    if tb:
        wv = b.transpose(wv, [1, 0])
    g = b.finish(b.matmul(av, wv))
    gen = torch.Generator().manual_seed(3)
    if kind == "f32":
        feeds = {"a": torch.randn(ash, generator=gen), "b": torch.randn(bsh, generator=gen)}
    else:
        feeds = {"a": torch.randint(-128, 128, ash, generator=gen, dtype=torch.int8),
                 "b": torch.randint(-128, 128, bsh, generator=gen, dtype=torch.int8)}
    _, (out,) = run(g, feeds)
    ref = interp.run(g, feeds)[0]
    if kind == "f32":
        assert rel_err(out, ref) < TF32_TOL
    else:
        assert torch.equal(out, ref)


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("kind", ["f32", "i8"])
def test_pair_gemm_layouts(cuda, ta, tb, kind):
    """Whole 256 x 256 tiles run on SM pairs (tcgen05 cta_group::2): every operand major, ragged K."""
    M, N, K = 512, 768, 96 if kind == "f32" else 320
    b = ir.Builder()
    ash, bsh = ([K, M] if ta else [M, K]), ([N, K] if tb else [K, N])
    dt = ir.FLOAT32 if kind == "f32" else ir.INT8
    a = b.input(ash, dt, name="a")
    w = b.input(bsh, dt, name="b")
    av, wv = (a, w) if kind == "f32" else (b.cast(a, ir.INT32), b.cast(w, ir.INT32))
    if ta:
        av = b.transpose(av, [1, 0])
    if tb:
        wv = b.transpose(wv, [1, 0])
    g = b.finish(b.relu(b.matmul(av, wv)) if kind == "f32" else b.matmul(av, wv))
    from tgcb import runtime

    assert all(ln.pair for s in runtime.generate(g)[3].steps if s.kind == "gemm" for ln in s.launches)
    gen = torch.Generator().manual_seed(5)
    if kind == "f32":
        feeds = {"a": torch.randn(ash, generator=gen), "b": torch.randn(bsh, generator=gen)}
    else:
        feeds = {"a": torch.randint(-128, 128, ash, generator=gen, dtype=torch.int8),
                 "b": torch.randint(-128, 128, bsh, generator=gen, dtype=torch.int8)}
    _, (out,) = run(g, feeds)
    ref = interp.run(g, feeds)[0]
    if kind == "f32":
        assert rel_err(out, ref) < TF32_TOL
    else:
        assert torch.equal(out, ref)


def test_simt_fallback_gemm(cuda):
    b = ir.Builder()
    a = b.input([5, 3], name="a")
    w = b.input([3, 7], name="w")
    g = b.finish(b.relu(b.matmul(a, w)))
    feeds = {"a": torch.randn(5, 3), "w": torch.randn(3, 7)}
    _, (out,) = run(g, feeds)
    assert rel_err(out, interp.run(g, feeds)[0]) < TF32_TOL


def test_int8_linear_full_size_bit_exact(cuda):
    """Quantise on the GPU, int8 GEMM with int32 accumulation, fused dequant: all bit-exact to tgc."""
    from tgcb import quantize

    with open(os.path.join(GOLDEN, "int8.json")) as f:
        meta = json.load(f)
    gold = np.load(os.path.join(GOLDEN, "int8.npz"))
    ins = workloads.int8_inputs()
    qa, sa = quantize.quantise_rows(ins["a"].cuda())
    qwt, sw = quantize.quantise_rows(ins["w"].T.contiguous().cuda())
    assert sha(qa) == meta["qa_sha"] and sha(qwt) == meta["qwt_sha"]
    assert np.array_equal(sa.cpu().numpy(), gold["sa"].reshape(-1))
    assert np.array_equal(sw.cpu().numpy(), gold["sw"].reshape(-1))
    g = workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32)
    c = compile_graph(g)
    acc, y = c({"qa": qa, "qwt": qwt, "sa": sa.reshape(-1, 1), "sw": sw.reshape(1, -1)})
    torch.cuda.synchronize()
    c.check_status()
    assert sha(acc) == meta["acc_sha"]
    assert sha(y) == meta["y_sha"]


def test_gradient_graph_matches_tgc(cuda):
    gold = np.load(os.path.join(GOLDEN, "train.npz"))
    g = load_graph("train_grad_small")
    feeds = {v.name: torch.from_numpy(gold[f"in/{v.name}"]) for v in g.inputs}
    _, out = run(g, feeds)
    for i, o in enumerate(out):
        assert rel_err(o, torch.from_numpy(gold[f"grad_opt/{i}"])) < TF32_TOL


def test_column_full_and_generic_reductions(cuda):
    b = ir.Builder()
    x = b.input([300, 77], name="x")
    y = b.input([4, 5, 6], name="y")
    g = b.finish(b.sum(x, [0]), b.max(x, [0], keepdims=True), b.sum(x, [0, 1]), b.mean(y, [0, 2]), b.sum(y, [1]))
    gen = torch.Generator().manual_seed(9)
    feeds = {"x": torch.randn(300, 77, generator=gen), "y": torch.randn(4, 5, 6, generator=gen)}
    c, out = run(g, feeds)
    ref = interp.run(g, feeds)
    for o, r in zip(out, ref, strict=True):
        assert o.shape == r.shape
        assert rel_err(o, r) < F32_RTOL
    col = next(s for s in c.module.steps if s.kind == "colreduce")
    rows_per_part = int(col.bracketing.split("blocks of ")[1].split()[0])
    assert np.array_equal(out[0].numpy(), bracketing.col_parts(feeds["x"].numpy(), rows_per_part))


def test_integer_reductions_exact(cuda):
    """int8 sums widen to int32 (accumulator_for, tgc/ir/dtype.py:139-151); int32 row, column and
    full sums and maxima are exact, so they must equal the interpreter's bit for bit. (tgc's
    interpreter hands back torch's int64 for integer sums; values are compared in the graph's
    declared int32, with inputs small enough that no int32 sum wraps.)"""
    b = ir.Builder()
    q = b.input([64, 300], ir.INT8, name="q")
    n = b.input([257, 33], ir.INT32, name="n")
    g = b.finish(b.sum(q, [1]), b.sum(q, [0]), b.sum(n, [0]), b.max(n, [1]), b.sum(n, [0, 1]))
    gen = torch.Generator().manual_seed(11)
    feeds = {"q": torch.randint(-128, 128, (64, 300), generator=gen, dtype=torch.int8),
             "n": torch.randint(-(1 << 16), 1 << 16, (257, 33), generator=gen, dtype=torch.int32)}
    _, out = run(g, feeds)
    ref = interp.run(g, feeds)
    for o, r in zip(out, ref, strict=True):
        assert o.dtype == torch.int32 and o.shape == r.shape
        assert torch.equal(o, r.to(torch.int32))


def test_views_and_broadcasts(cuda):
    b = ir.Builder()
    x = b.input([6, 8], name="x")
    v = b.input([8], name="v")
    t = b.transpose(x, [1, 0])
    r = b.reshape(t, [4, 12])
    s = b.slice(r, 1, 2, 5)
    cat = b.concat(s, b.neg(s), axis=1)
    z = b.add(x, b.broadcast_to(v, [6, 8]))
    g = b.finish(cat, b.sigmoid(z), b.cast(b.step(z), ir.INT32))
    gen = torch.Generator().manual_seed(2)
    feeds = {"x": torch.randn(6, 8, generator=gen), "v": torch.randn(8, generator=gen)}
    _, out = run(g, feeds)
    ref = interp.run(g, feeds)
    assert torch.equal(out[0], ref[0])
    assert rel_err(out[1], ref[1]) < F32_RTOL
    assert torch.equal(out[2], ref[2])


def test_host_feeds_and_missing_inputs(cuda):
    g = workloads.cone_graph(ir.Builder, rows=64, cols=256)
    feeds = workloads.cone_inputs(rows=64, cols=256)
    c = compile_graph(g)
    host = c(feeds)  # CPU tensors are copied into their planned slots
    dev = c(on_gpu(feeds))
    torch.cuda.synchronize()
    for a, b in zip(host, dev, strict=True):
        assert torch.equal(a, b)
    with pytest.raises(ConfigError, match="no value supplied"):
        c({})


def test_outputs_are_views_of_the_arena(cuda):
    """tgc's contract (emit.py:201-202): outputs live in the arena; the next call overwrites them."""
    g = workloads.cone_graph(ir.Builder, rows=16, cols=64)
    c = compile_graph(g)
    arena = c.new_arena()
    f1 = on_gpu(workloads.cone_inputs(rows=16, cols=64, seed=1))
    f2 = on_gpu(workloads.cone_inputs(rows=16, cols=64, seed=2))
    first = c.function(arena, f1)[0]
    keep = first.clone()
    second = c.function(arena, f2)[0]
    torch.cuda.synchronize()
    assert first.data_ptr() == second.data_ptr()
    assert not torch.equal(first, keep)
