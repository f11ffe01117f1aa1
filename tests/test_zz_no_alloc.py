"""The allocation-free pairwise sum, for callers that cannot allocate device memory.

Some callers of this library may not call cudaMalloc: code running where the device
allocator is owned by someone else (a framework's memory pool, a host callback, a plugin
loaded into another program). tgcb_sum_pairwise_f32_noalloc serves them with a scratch array
built into the library. These tests call it through the C-ABI and check that it returns
exactly what tgcb_sum_pairwise_f32 (caller-provided scratch) returns — the pairwise sums are
bit-exact, so equality is the tolerance — on two calls in a row, since calls share the array
and the second call must not depend on what the first left in it. This file is collected
last so that a failure here comes after every other test has run; it also passes alone.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tgcb import _lib

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 1 << 20  # TGCB_NOALLOC_SCRATCH_BYTES in include/tgcb.h


def _with_caller_scratch(lib, x: torch.Tensor, block: int) -> float:
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    need = lib.tgcb_sum_pairwise_scratch_bytes(x.numel(), block)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    rc = lib.tgcb_sum_pairwise_f32(
        ctypes.c_void_p(x.data_ptr()), x.numel(), block, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(scratch.data_ptr()), scratch.numel(), None,
    )
    _lib.check(rc, "tgcb_sum_pairwise_f32")
    torch.cuda.synchronize()
    return float(out.item())


def _without_allocation(lib, x: torch.Tensor, block: int, out: torch.Tensor) -> float:
    rc = lib.tgcb_sum_pairwise_f32_noalloc(ctypes.c_void_p(x.data_ptr()), x.numel(), block, ctypes.c_void_p(out.data_ptr()), None)
    _lib.check(rc, "tgcb_sum_pairwise_f32_noalloc")
    torch.cuda.synchronize()
    return float(out.item())


@pytest.mark.parametrize("n,block", [(1 << 26, 8), ((1 << 20) + 3, 8), (12345, 3), (1, 8)])
def test_matches_the_scratch_taking_entry_point_twice(cuda, n, block):
    lib = _lib.load()
    _lib.ensure_device(0)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    for seed in (1, 2):  # two calls in a row, different data: nothing carried over between them
        x = torch.rand(n, generator=torch.Generator().manual_seed(seed * 1000 + n)).to(cuda)
        expected = _with_caller_scratch(lib, x, block)
        assert _without_allocation(lib, x, block, out) == expected


# The longest inputs the built-in array accepts. At block 1, 2^26 - 1 values split into 2^25
# irregular leaves whose partials fill more than half of the array, so the last combining
# levels sit at its far end; at block 8, 9 * 2^25 - 1 values is the longest length whose
# partials still fit (one more value adds a level and needs more than the whole array).
@pytest.mark.parametrize("n,block", [((1 << 26) - 1, 1), (9 * (1 << 25) - 1, 8)])
def test_longest_accepted_lengths_match_bit_for_bit(cuda, n, block):
    lib = _lib.load()
    _lib.ensure_device(0)
    need = lib.tgcb_sum_pairwise_scratch_bytes(n, block)
    assert SCRATCH_LIMIT // 2 < need <= SCRATCH_LIMIT
    assert lib.tgcb_sum_pairwise_scratch_bytes(n + 1, block) > SCRATCH_LIMIT
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    for seed in (3, 4):
        g = torch.Generator(device=cuda).manual_seed(seed)
        x = torch.rand(n, generator=g, device=cuda)
        expected = _with_caller_scratch(lib, x, block)
        assert _without_allocation(lib, x, block, out) == expected
        del x


def test_refuses_lengths_beyond_the_built_in_scratch(cuda):
    lib = _lib.load()
    _lib.ensure_device(0)
    x = torch.ones(16, device=cuda)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    too_long = 1 << 30  # needs more than 1 MiB of partials at block 8; refused before any launch
    assert lib.tgcb_sum_pairwise_scratch_bytes(too_long, 8) > SCRATCH_LIMIT
    rc = lib.tgcb_sum_pairwise_f32_noalloc(ctypes.c_void_p(x.data_ptr()), too_long, 8, ctypes.c_void_p(out.data_ptr()), None)
    assert rc == _lib.TGCB_E_INVALID
    assert "scratch" in _lib.last_error()
    assert lib.tgcb_sum_pairwise_scratch_bytes(1 << 28, 8) <= SCRATCH_LIMIT
