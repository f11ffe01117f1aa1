"""Two GEMMs in one chain launch against the same graph as two launches and against the oracle.

A chain runs the same tiles with the same k-order and the same epilogues as the two separate
SM-pair launches, so its outputs must be bit-identical to theirs; both are also checked
against the oracle at the TF32 tolerance of the GEMM tests (5e-3 of the largest output).
"""

from __future__ import annotations

import pytest
import torch

from oracle import interp
from tgcb import codegen, ir
from tgcb.runtime import compile_graph

pytestmark = pytest.mark.gpu


def mlp_like(rows, k, n1, n2, act="gelu"):
    b = ir.Builder()
    x = b.input((rows, k), ir.FLOAT32, "x")
    w1 = b.input((k, n1), ir.FLOAT32, "w1")
    b1 = b.input((n1,), ir.FLOAT32, "b1")
    w2 = b.input((n1, n2), ir.FLOAT32, "w2")
    h = b.add(b.matmul(x, w1), b1)
    h = b.relu(h) if act == "relu" else b.tanh(h)
    return b.finish(b.matmul(h, w2))


def feeds(g, seed):
    return interp.random_feeds(g, seed=seed, positive=False)


def run(g, f, chained: bool, monkeypatch):
    monkeypatch.setattr(codegen, "CHAIN_GEMM", chained)
    # the two launches run their GEMMs whole, as the chain does (a K split would change the
    # order of the fp32 additions)
    monkeypatch.setattr(codegen, "K_SPLIT", False)
    c = compile_graph(g)
    kinds = [ln.gemm2 is not None for s in c.module.steps for ln in s.launches if ln.gemm]
    assert any(kinds) == chained
    out = [o.clone() for o in c({k: v.cuda() for k, v in f.items()})]
    torch.cuda.synchronize()
    c.check_status()
    return c, out


@pytest.mark.parametrize(
    "rows,k,n1,n2",
    [
        (512, 256, 512, 256),     # 4 + 2 tiles: most pairs have nothing to do
        (2048, 128, 1024, 512),   # 32 + 16 tiles
        (8192, 1024, 4096, 1024), # the MLP block's shapes: 512 + 128 tiles
        (4096, 64, 256, 768),     # one k-block in the first GEMM, 16 + 48 tiles
    ],
)
def test_chain_is_bit_identical_to_two_launches(cuda, monkeypatch, rows, k, n1, n2):
    g = mlp_like(rows, k, n1, n2)
    f = feeds(g, 3)
    _, two = run(g, f, False, monkeypatch)
    _, one = run(g, f, True, monkeypatch)
    for a, b in zip(one, two, strict=True):
        assert torch.equal(a, b)
    if rows <= 2048:
        (want,) = interp.run(g, f)
        got = one[0].cpu().double()
        assert float((got - want.double()).abs().max()) <= 5e-3 * float(want.double().abs().max())


def test_chain_counters_are_fresh_every_call(cuda, monkeypatch):
    # a launch that found stale counters would let second-GEMM tiles read rows not yet written
    g = mlp_like(2048, 256, 1024, 256, act="relu")
    monkeypatch.setattr(codegen, "CHAIN_GEMM", True)
    c = compile_graph(g)
    arena = c.new_arena()
    for seed in range(1, 6):
        f = feeds(g, seed)
        got = c.function(arena, {k: v.cuda() for k, v in f.items()})[0].clone()
        torch.cuda.synchronize()
        (want,) = interp.run(g, f)
        assert float((got.cpu().double() - want.double()).abs().max()) <= 5e-3 * float(want.double().abs().max()), seed
    c.check_status()


def test_chain_on_two_arenas_and_streams(cuda, monkeypatch):
    g = mlp_like(2048, 256, 1024, 256)
    monkeypatch.setattr(codegen, "CHAIN_GEMM", True)
    c = compile_graph(g)
    arenas = [c.new_arena(), c.new_arena()]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    fs = [feeds(g, 10 + i) for i in range(4)]
    outs = []
    for i, f in enumerate(fs):
        s = streams[i % 2]
        with torch.cuda.stream(s):
            o = c.function(arenas[i % 2], {k: v.cuda() for k, v in f.items()}, stream=s)[0]
            outs.append(o.clone())
    torch.cuda.synchronize()
    c.check_status()
    for f, got in zip(fs, outs, strict=True):
        (want,) = interp.run(g, f)
        assert float((got.cpu().double() - want.double()).abs().max()) <= 5e-3 * float(want.double().abs().max())


@pytest.mark.parametrize(
    "rows,d,f",
    [
        (512, 256, 512),     # 32 row groups for 148 CTAs: most CTAs compute no rows
        (2048, 256, 1024),
        (8192, 1024, 4096),  # the MLP block
    ],
)
def test_layernorm_prologue_is_bit_identical_to_its_own_launch(cuda, monkeypatch, rows, d, f):
    # the layernorm rows computed by the chain's epilogue warps run the row kernel's code for
    # one warp per row, so every output matches the separate row-kernel launch bit for bit
    from tgcb import workloads

    g = workloads.mlp_graph(ir.Builder, rows=rows, d=d, f=f)
    f_in = workloads.mlp_inputs(rows=rows, d=d, f=f, seed=5)
    outs = {}
    for pro in (False, True):
        monkeypatch.setattr(codegen, "ROW_PROLOGUE", pro)
        monkeypatch.setattr(codegen, "CHAIN_GEMM", True)
        c = compile_graph(g)
        kinds = [s.kind for s in c.module.steps]
        assert kinds == (["gemm"] if pro else ["row", "gemm"])
        arena = c.new_arena()
        for _ in range(2):  # the second call reuses the arena and the counters
            got = [o.clone() for o in c.function(arena, {k: v.cuda() for k, v in f_in.items()})]
        torch.cuda.synchronize()
        c.check_status()
        outs[pro] = got
    for a, b in zip(outs[True], outs[False], strict=True):
        assert torch.equal(a, b)
    if rows <= 2048:
        (want,) = interp.run(g, f_in)
        got = outs[True][0].cpu().double()
        assert float((got - want.double()).abs().max()) <= 5e-3 * float(want.double().abs().max())
