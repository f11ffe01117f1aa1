"""SM-pair GEMMs with K cut into slices (fewer output tiles than SM pairs: the training step's
weight gradients) against the same GEMM unsplit and against the oracle.

The slices of every 32 x 64 region are summed in slice order by whichever slice finishes last,
so a split GEMM gives the same bits on every run; int8 partials are int32 and exact, so the
int8 split equals the oracle bit for bit. TF32 results differ from the unsplit GEMM only by
the order of the fp32 additions of the slices: both are checked at 5e-3 of the largest output.
"""

from __future__ import annotations

import pytest
import torch

from oracle import interp
from tgcb import codegen, ir, workloads
from tgcb.runtime import compile_graph

pytestmark = pytest.mark.gpu


def weight_gradient(rows, m, n):
    # dW = X^T @ dY, as the training step's reverse pass writes it: both operands MN-major
    b = ir.Builder()
    x = b.input((rows, m), ir.FLOAT32, "x")
    dy = b.input((rows, n), ir.FLOAT32, "dy")
    return b.finish(b.matmul(b.transpose(x, [1, 0]), dy))


def linear(rows, k, n):
    b = ir.Builder()
    x = b.input((rows, k), ir.FLOAT32, "x")
    w = b.input((k, n), ir.FLOAT32, "w")
    return b.finish(b.matmul(x, w))


def run(g, feeds, split: bool, monkeypatch, times=1):
    monkeypatch.setattr(codegen, "K_SPLIT", split)
    c = compile_graph(g)
    counters = [ln.counter_bytes for s in c.module.steps for ln in s.launches if ln.gemm]
    assert (max(counters) > 0) == split
    outs = []
    for _ in range(times):
        outs.append([o.clone() for o in c({k: v.cuda() for k, v in feeds.items()})])
        torch.cuda.synchronize()
    c.check_status()
    return outs


def close(a, b):
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return float((a - b).abs().max()) <= 5e-3 * float(b.abs().max())


@pytest.mark.parametrize(
    "make,args",
    [
        (weight_gradient, (16384, 1024, 1024)),  # 16 output tiles, 512 k-blocks: 4 slices
        (weight_gradient, (8192, 512, 768)),     # 6 tiles
        (linear, (512, 8192, 512)),              # 4 tiles, K-major A
    ],
)
def test_split_gemm_matches_unsplit_and_oracle(cuda, monkeypatch, make, args):
    g = make(*args)
    feeds = interp.random_feeds(g, seed=7)
    (one,), = run(g, feeds, False, monkeypatch)
    runs = run(g, feeds, True, monkeypatch, times=3)
    for other in runs[1:]:
        assert torch.equal(runs[0][0], other[0])  # the same bits on every call
    assert close(runs[0][0], one)
    (want,) = interp.run(g, feeds)
    assert close(runs[0][0], want)


def test_int8_split_is_exact(cuda, monkeypatch):
    # int32 partials add exactly: the split GEMM equals the oracle's exact integer GEMM
    g = workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32, rows=512, k=16384, n=512)
    gen = torch.Generator().manual_seed(3)
    feeds = {
        "qa": torch.randint(-128, 128, (512, 16384), generator=gen, dtype=torch.int8),
        "qwt": torch.randint(-128, 128, (512, 16384), generator=gen, dtype=torch.int8),
        "sa": torch.rand(512, 1, generator=gen),
        "sw": torch.rand(1, 512, generator=gen),
    }
    (acc, y), = run(g, feeds, True, monkeypatch)
    want = feeds["qa"].double() @ feeds["qwt"].double().t()
    assert torch.equal(acc.cpu().double(), want)
