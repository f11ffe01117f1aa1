"""tgc's executor tests (tests/test_executor.py: TestExecution) re-pointed at the B200 backend:
every graph of its GRAPHS table and the transpose pair/chain of passes/layout.py, printed by
tgc (tests/golden/graphs/exec_*.tgc), compiled with and without the pass pipeline, checked
against the oracle on the same seeded feeds, then run again on one arena with seeds 1-7
(a kernel that reads a buffer before writing it passes the first call and fails later).
Tolerance: rtol = atol = 1e-5 for float32 graphs, 5e-3 of the largest output for graphs with
a TF32 GEMM (tgc holds its own compiled path bit-identical to its interpreter because both are
torch on the CPU; here the arithmetic is the GPU's)."""

from __future__ import annotations

import ctypes
import os

import pytest
import torch
from conftest import GOLDEN

from oracle import interp
from tgcb import _lib, serialize
from tgcb.errors import AllocationError, ConfigError
from tgcb.runtime import compile_graph

pytestmark = pytest.mark.gpu

NAMES = ["chain", "softmax", "layernorm", "mlp", "diamond", "branching", "transposed_pair", "transposed_chain"]


def load(name):
    with open(os.path.join(GOLDEN, "graphs", f"exec_{name}.tgc")) as f:
        return serialize.loads(f.read())


def agree(got, want, gemm: bool) -> bool:
    for a, b in zip(got, want, strict=True):
        a = a.detach().cpu()
        if a.shape != b.shape:
            return False
        if gemm:
            if float((a.double() - b.double()).abs().max()) > 5e-3 * float(b.double().abs().max()):
                return False
        elif not torch.allclose(a.float(), b.float(), rtol=1e-5, atol=1e-5):
            return False
    return True


@pytest.mark.parametrize("optimise", [True, False], ids=["pipeline", "no_pipeline"])
@pytest.mark.parametrize("name", NAMES)
def test_every_executor_graph_matches(cuda, name, optimise):
    g = load(name)
    gemm = any(n.op.name == "matmul" for n in g.nodes)
    compiled = compile_graph(g, optimise=optimise)
    feeds = interp.random_feeds(g, seed=0, positive=True)
    out = compiled({k: v.cuda() for k, v in feeds.items()})
    torch.cuda.synchronize()
    compiled.check_status()
    assert agree(out, interp.run(g, feeds), gemm), name


@pytest.mark.parametrize("name", NAMES)
def test_the_arena_survives_reuse(cuda, name):
    g = load(name)
    gemm = any(n.op.name == "matmul" for n in g.nodes)
    compiled = compile_graph(g)
    arena = compiled.new_arena()
    for seed in range(1, 8):
        feeds = interp.random_feeds(g, seed=seed, positive=True)
        out = [o.clone() for o in compiled.function(arena, {k: v.cuda() for k, v in feeds.items()})]
        torch.cuda.synchronize()
        assert agree(out, interp.run(g, feeds), gemm), (name, seed)
    compiled.check_status()


def test_a_missing_input_is_reported(cuda):
    compiled = compile_graph(load("softmax"))
    with pytest.raises(ConfigError, match="no value supplied"):
        compiled({})


def test_a_short_or_null_input_table_is_refused_before_any_launch(cuda):
    """A C caller of tgcb_plan_run gets TGCB_E_INVALID, not a kernel reading through a null
    pointer, when its input table is short or holds a null entry; the plan still runs after."""
    graph = load("mlp")
    compiled = compile_graph(graph)
    assert len(compiled.input_names) > 1
    feeds = interp.random_feeds(graph, seed=0, positive=True)
    arena = compiled.new_arena()
    ptrs = compiled.input_pointers(arena, {n: t.to(cuda) for n, t in feeds.items()})
    torch.cuda.synchronize()
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    short = (ctypes.c_void_p * len(ptrs))(*ptrs)
    rc = lib.tgcb_plan_run(compiled._plan, ctypes.c_void_p(arena.data_ptr()), short, len(ptrs) - 1, stream)
    assert rc == _lib.TGCB_E_INVALID and "the plan reads" in _lib.last_error()
    holed = (ctypes.c_void_p * len(ptrs))(*ptrs)
    holed[len(ptrs) - 1] = None
    rc = lib.tgcb_plan_run(compiled._plan, ctypes.c_void_p(arena.data_ptr()), holed, len(ptrs), stream)
    assert rc == _lib.TGCB_E_INVALID and "null pointer" in _lib.last_error()
    with pytest.raises(AllocationError, match="the plan reads"):
        _lib.check(lib.tgcb_plan_run(compiled._plan, ctypes.c_void_p(arena.data_ptr()), short, 0, stream), "run")
    compiled.check_status()  # nothing was launched by the refused calls
    got = compiled.function(arena, {n: t.to(cuda) for n, t in feeds.items()})
    assert agree(got, interp.run(graph, feeds), gemm=True)


def test_descriptors_outside_the_arena_are_refused(cuda):
    """tgcb_plan_create checks every GEMM operand and counter range against the arena, also for
    sizes whose byte count would wrap around 64 bits; nothing is launched."""
    compiled = compile_graph(load("mlp"))
    lib = _lib.load()
    gemm = next(d for d in compiled.module.launches if d.is_gemm)

    def create(edit) -> int:
        d = _lib.LaunchDesc()
        ctypes.pointer(d)[0] = gemm
        edit(d)
        plan = ctypes.c_void_p()
        rc = lib.tgcb_plan_create(compiled._module, (_lib.LaunchDesc * 1)(d), 1, compiled.arena_bytes, ctypes.byref(plan))
        if rc == _lib.TGCB_OK:
            lib.tgcb_plan_destroy(plan)
        return rc

    def arena_operand(offset, rows, cols):
        def edit(d):
            d.a.input_index, d.a.arena_offset, d.a.rows, d.a.cols = -1, offset, rows, cols
        return edit

    assert create(lambda d: None) == _lib.TGCB_OK
    assert create(arena_operand(compiled.arena_bytes, 1, 1)) == _lib.TGCB_E_INVALID
    assert "outside the arena" in _lib.last_error()
    assert create(arena_operand(0, 1 << 40, 1 << 40)) == _lib.TGCB_E_INVALID  # 2^80 * 4 bytes wraps
    assert create(arena_operand((1 << 64) - 16, 1, 8)) == _lib.TGCB_E_INVALID  # offset + size wraps

    def counters(offset, nbytes):
        def edit(d):
            d.counter_offset, d.counter_bytes = offset, nbytes
        return edit

    assert create(counters((1 << 64) - 4, 8)) == _lib.TGCB_E_INVALID
    assert create(counters(0, compiled.arena_bytes + 4)) == _lib.TGCB_E_INVALID
    assert create(counters(0, 256)) == _lib.TGCB_OK
