"""The ahead-of-time kernels through the C-ABI: bit-exact float32 summation orders and the
per-row int8 quantiser, against tgc's golden values and the oracle's restatements."""

from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import bracketing
from oracle import quantize as oq
from tgcb import _lib, quantize, summation, workloads
from tgcb.errors import ConfigError

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def summ():
    with open(os.path.join(GOLDEN, "summation.json")) as f:
        return json.load(f)


def test_long_sum_bit_exact_to_tgc(cuda, summ):
    """2^26 values with a 1e8 leader: pairwise and sequential equal tgc's own results."""
    ls = summ["longsum"]
    v, idx = workloads.longsum_input()
    assert idx == ls["leader_index"]
    vc = v.cuda()
    p = summation.pairwise(vc)
    s = summation.sequential(vc)
    assert p == ls["pairwise"]
    assert s == ls["sequential"]
    exact = ls["exact"]
    # the point of the bracketing: the tree is orders of magnitude closer to the exact sum
    assert abs(p - exact) / exact < abs(s - exact) / exact


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_long_sum_in_shards_bit_exact_to_tgc(cuda, summ, shards):
    """The 2^26 sum split into depth-k subtrees (one per rank), each summed by the kernels and
    the partials combined by tgcb_sum_perfect_tree_f32: tgc's pairwise value, bit for bit."""
    v, _ = workloads.longsum_input()
    vc = v.cuda()
    parts = torch.empty(shards, dtype=torch.float32, device="cuda")
    for j, (a, b) in enumerate(summation.shard_ranges(v.numel(), shards)):
        scratch = torch.empty(summation.scratch_bytes(b - a), dtype=torch.uint8, device="cuda")
        summation.pairwise_into(vc[a:b], parts[j:j + 1], scratch)
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    summation.perfect_tree_into(parts, out)
    assert float(out.item()) == summ["longsum"]["pairwise"]


@pytest.mark.parametrize("count", [1, 2, 8, 64, 256])
def test_perfect_tree(cuda, count):
    p = torch.rand(count, generator=torch.Generator().manual_seed(count)) * 1e4 - 3e3
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    summation.perfect_tree_into(p.cuda(), out)
    want = [np.float32(x) for x in p.numpy()]
    while len(want) > 1:
        want = [np.float32(want[i] + want[i + 1]) for i in range(0, len(want), 2)]
    assert float(out.item()) == float(want[0])


@pytest.mark.parametrize("count", [3, 512])
def test_perfect_tree_refuses(cuda, count):
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    ones = torch.ones(count, device="cuda")
    with pytest.raises(ConfigError):
        summation.perfect_tree_into(ones, out)
    rc = _lib.load().tgcb_sum_perfect_tree_f32(ctypes.c_void_p(ones.data_ptr()), count, ctypes.c_void_p(out.data_ptr()), None)
    assert rc == _lib.TGCB_E_INVALID and "power of two" in _lib.last_error()


def test_summation_vectors_bit_exact_to_tgc(cuda, summ):
    gens = {
        "uniform": lambda c, s: np.asarray(np.random.default_rng(s).uniform(0.5, 1.5, size=c), dtype=np.float32),
        "mixed": lambda c, s: np.asarray([1e9, *np.random.default_rng(s).uniform(0.5, 1.5, size=c - 1)], dtype=np.float32),
        "alternating": lambda c, s: np.asarray(np.random.default_rng(s).normal(0.0, 1.0, size=c), dtype=np.float32),
    }
    for vec in summ["vectors"]:
        v = torch.from_numpy(gens[vec["kind"]](vec["count"], vec["seed"])).cuda()
        assert summation.sequential(v) == vec["sequential"]
        assert summation.pairwise(v) == vec["pairwise"]
        assert summation.pairwise(v, block=3) == vec["pairwise_block_3"]


@pytest.mark.parametrize(
    "n", [1, 2, 7, 8, 9, 17, 255, 256, 257, 1000, 4096, 12345, 65537, 196608, 1000003, (1 << 21) + 3, 3 << 20, 1 << 22, 1 << 24]
)
@pytest.mark.parametrize("block", [1, 3, 8, 16])
def test_pairwise_any_length_any_block(cuda, n, block):
    v = torch.rand(n, generator=torch.Generator().manual_seed(n + block)) - 0.3
    assert summation.pairwise(v.cuda(), block) == bracketing.pairwise(v.numpy(), block)


@pytest.mark.parametrize("n", [1, 5, 1000, 65535, 65537, 2048 * 16 * 3 + 7])
def test_sequential_any_length(cuda, n):
    v = torch.rand(n, generator=torch.Generator().manual_seed(n))
    assert summation.sequential(v.cuda()) == bracketing.sequential(v.numpy())


@pytest.mark.parametrize("offset", [1, 2, 3])
@pytest.mark.parametrize("n", [70001, (1 << 20) + 5])
def test_sequential_on_unaligned_views(cuda, n, offset):
    """Long vectors stream through shared memory in 16-byte-aligned bulk copies; a view that
    starts 4, 8 or 12 bytes past a 16-byte boundary adds its head and ragged tail directly, in
    the same left-to-right order."""
    v = torch.rand(n, generator=torch.Generator().manual_seed(n + offset)) - 0.25
    vc = v.cuda()[offset:]
    assert vc.data_ptr() % 16 != 0
    assert summation.sequential(vc) == bracketing.sequential(v.numpy()[offset:])


@pytest.mark.parametrize("n", [4099, (1 << 20) + 3])
def test_pairwise_on_an_unaligned_view(cuda, n):
    v = torch.rand(n, generator=torch.Generator().manual_seed(1))
    vc = v.cuda()[3:]
    assert summation.pairwise(vc) == bracketing.pairwise(v.numpy()[3:])


def test_summation_input_checks(cuda):
    with pytest.raises(ConfigError, match="nothing to sum"):
        summation.pairwise(torch.empty(0, device="cuda"))
    with pytest.raises(ConfigError, match="float32"):
        summation.sequential(torch.ones(4, dtype=torch.float64, device="cuda"))
    with pytest.raises(ConfigError, match="vector"):
        summation.pairwise(torch.ones(2, 2, device="cuda"))


def test_pairwise_rejects_short_scratch(cuda):
    lib = _lib.load()
    v = torch.ones(1 << 16, device="cuda")
    out = torch.empty(1, device="cuda")
    rc = lib.tgcb_sum_pairwise_f32(ctypes.c_void_p(v.data_ptr()), v.numel(), 8, ctypes.c_void_p(out.data_ptr()),
                                   ctypes.c_void_p(out.data_ptr()), 4, None)
    assert rc == _lib.TGCB_E_INVALID
    assert "scratch" in _lib.last_error()


def test_quantiser_bit_exact_to_tgc(cuda):
    gold = np.load(os.path.join(GOLDEN, "quantize.npz"))
    for name in ("randn", "weights_t", "edge"):
        x = torch.from_numpy(gold[f"{name}/x"]).cuda()
        q, s = quantize.quantise_rows(x)
        assert np.array_equal(q.cpu().numpy().astype(np.float32), gold[f"{name}/q"])
        assert np.array_equal(s.cpu().numpy(), gold[f"{name}/scale"].astype(np.float32))


@pytest.mark.parametrize("rows,cols", [(3, 1), (17, 1000), (64, 4096), (5, 5000), (8, 1024), (4, 2048), (3, 3072), (2, 8192), (2, 16384)])
def test_quantiser_shapes(cuda, rows, cols):
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(cols)) * 3
    q, s = quantize.quantise_rows(x.cuda())
    qo, so = oq.quantise_rows(x.numpy())
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)


@pytest.mark.parametrize("m", [127.0, 12.7, 3.0, 1e-3])
def test_quantiser_ties(cuda, m):
    """Values whose quotient by the row scale sits on or next to a half-integer: the fast
    reciprocal path must hand those to the exact quotient (round half to even)."""
    s = np.float32(m / 127.0)
    k = np.arange(-127, 127, dtype=np.float32)
    on = (k + np.float32(0.5)) * s
    near = np.concatenate([on, np.nextafter(on, np.float32(np.inf)), np.nextafter(on, np.float32(-np.inf))])
    row = np.concatenate([[np.float32(m)], near, np.zeros(1024 - 1 - near.size % 1024, dtype=np.float32)])
    row = row[: (row.size // 1024) * 1024].astype(np.float32)
    x = np.tile(row, (3, 1))
    q, sc = quantize.quantise_rows(torch.from_numpy(x).cuda())
    qo, so = oq.quantise_rows(x)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(sc.cpu().numpy(), so)


def test_quantiser_input_checks(cuda):
    with pytest.raises(ConfigError):
        quantize.quantise_rows(torch.ones(4, device="cuda"))
    with pytest.raises(ConfigError):
        quantize.quantise_rows(torch.ones(0, 3, device="cuda"))


def test_device_status_stays_clear(cuda):
    st = ctypes.c_int(-1)
    _lib.check(_lib.load().tgcb_status(1, ctypes.byref(st)), "tgcb_status")
    assert st.value == 0
