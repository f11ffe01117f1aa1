"""float32 summation orders on the GPU, bit-exact to tgc/analysis/summation.py.

``pairwise`` and ``sequential`` take a 1-D float32 CUDA tensor and return the same Python
float tgc's functions return for the same values (summation.py:56-85), computed by the
library's kernels (tgcb_sum_pairwise_f32, tgcb_sum_sequential_f32). The input checks and
their ``ConfigError`` messages follow tgc's ``_checked`` (summation.py:36-44).
``*_into`` variants write the result to a device scalar on a stream without synchronising.

Across GPUs the pairwise order shards without losing bit-exactness: for 2^k ranks each rank
holds one depth-k node of the halving (``shard_ranges``), sums it with the same kernels (a node's
_pairwise value depends only on its own values), and the 2^k partials, gathered in rank order,
are the leaves of the perfect tree that forms the top k levels (``tgcb_sum_perfect_tree_f32``).
``ShardedPairwise`` does that with one all-gather of one float per rank.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from tgcb import _lib
from tgcb.errors import ConfigError

DEFAULT_BLOCK = 8


def _checked(values: torch.Tensor) -> torch.Tensor:
    if not isinstance(values, torch.Tensor) or not values.is_cuda:
        raise ConfigError("the GPU orders take a CUDA tensor")
    if values.dim() != 1:
        raise ConfigError(f"a reduction runs over a vector, got rank {values.dim()}")
    if values.numel() == 0:
        raise ConfigError("there is nothing to sum")
    if values.dtype != torch.float32:
        raise ConfigError(f"these orders are about float32, got {values.dtype}")
    return values.contiguous()


def scratch_bytes(n: int, block: int = DEFAULT_BLOCK) -> int:
    return int(_lib.load().tgcb_sum_pairwise_scratch_bytes(n, block))


def pairwise_into(values: torch.Tensor, out: torch.Tensor, scratch: torch.Tensor, block: int = DEFAULT_BLOCK, stream=None) -> None:
    v = _checked(values)
    if block < 1:
        raise ConfigError(f"a block of {block} values is not a block")
    _lib.ensure_device(v.device.index)
    s = stream if stream is not None else torch.cuda.current_stream(v.device)
    rc = _lib.load().tgcb_sum_pairwise_f32(
        ctypes.c_void_p(v.data_ptr()), v.numel(), block, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(scratch.data_ptr()), scratch.numel() * scratch.element_size(), ctypes.c_void_p(s.cuda_stream),
    )
    _lib.check(rc, "tgcb_sum_pairwise_f32")


def sequential_into(values: torch.Tensor, out: torch.Tensor, stream=None) -> None:
    v = _checked(values)
    _lib.ensure_device(v.device.index)
    s = stream if stream is not None else torch.cuda.current_stream(v.device)
    rc = _lib.load().tgcb_sum_sequential_f32(
        ctypes.c_void_p(v.data_ptr()), v.numel(), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(s.cuda_stream)
    )
    _lib.check(rc, "tgcb_sum_sequential_f32")


def levels_for(n: int, block: int = DEFAULT_BLOCK) -> int:
    """Depth L of the perfect part of _pairwise's tree: the least L with n >> L <= block."""
    if n < 1 or block < 1:
        raise ConfigError(f"no pairwise tree over {n} values with blocks of {block}")
    levels = 0
    while (n >> levels) > block:
        levels += 1
    return levels


def subtree_range(n: int, depth: int, index: int) -> tuple[int, int]:
    """[start, stop) of node ``index`` at ``depth`` of _pairwise's halving of n values.

    A range of size s splits into its first s // 2 values and the rest (summation.py:81-84);
    bit ``depth-1-level`` of ``index`` says which half is taken at each level.
    """
    if not 0 <= index < (1 << depth):
        raise ConfigError(f"node {index} is outside depth {depth}")
    start, size = 0, n
    for level in range(depth - 1, -1, -1):
        half = size // 2
        if (index >> level) & 1:
            start, size = start + half, size - half
        else:
            size = half
    return start, start + size


def shard_ranges(n: int, shards: int, block: int = DEFAULT_BLOCK) -> list[tuple[int, int]]:
    """The contiguous ranges 2^k shards take so that their pairwise sums are depth-k nodes.

    Refuses a shard count that is not a power of two, or one deeper than the perfect part of
    the tree (a node there would be a leaf block, summed sequentially, not split).
    """
    if shards < 1 or shards & (shards - 1):
        raise ConfigError(f"the pairwise tree shards over a power of two, not {shards}")
    depth = shards.bit_length() - 1
    if shards > 1 and depth > levels_for(n, block):
        raise ConfigError(f"{n} values in blocks of {block} do not split {shards} ways inside the tree")
    if shards > 256:
        raise ConfigError("at most 256 shards are combined")
    return [subtree_range(n, depth, j) for j in range(shards)]


def perfect_tree_into(partials: torch.Tensor, out: torch.Tensor, stream=None) -> None:
    """((p0+p1)+(p2+p3))+... over a power-of-two count of float32 partials, on the GPU."""
    p = _checked(partials)
    if p.numel() > 256 or p.numel() & (p.numel() - 1):
        raise ConfigError(f"a perfect tree takes a power of two from 1 to 256 partials, not {p.numel()}")
    _lib.ensure_device(p.device.index)
    s = stream if stream is not None else torch.cuda.current_stream(p.device)
    rc = _lib.load().tgcb_sum_perfect_tree_f32(
        ctypes.c_void_p(p.data_ptr()), p.numel(), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(s.cuda_stream)
    )
    _lib.check(rc, "tgcb_sum_perfect_tree_f32")


class ShardedPairwise:
    """The pairwise sum of an n-value vector whose ``shard_ranges`` slices live one per rank.

    ``dist`` is ``torch.distributed`` (NCCL on GPUs); every rank calls ``into`` (or ``__call__``)
    with its own slice and gets the whole vector's sum, bit-exact to tgc's ``pairwise``.
    """

    def __init__(self, n: int, rank: int, world: int, dist, device, block: int = DEFAULT_BLOCK, *,
                 shard_sum=None, tree=None):
        """``shard_sum(local, out)`` and ``tree(partials, out)`` default to the library's kernels;
        tests on CPU ranks pass the oracle's orders instead."""
        self.ranges = shard_ranges(n, world, block)
        self.n, self.rank, self.world, self.dist, self.block = n, rank, world, dist, block
        start, stop = self.ranges[rank]
        self.local = stop - start
        self.partial = torch.empty(1, dtype=torch.float32, device=device)
        self.gathered = torch.empty(world, dtype=torch.float32, device=device)
        if shard_sum is None:
            scratch = torch.empty(max(1, scratch_bytes(self.local, block)), dtype=torch.uint8, device=device)
            shard_sum = lambda local, out: pairwise_into(local, out, scratch, block)  # noqa: E731
        self._shard_sum = shard_sum
        self._tree = tree if tree is not None else perfect_tree_into

    def into(self, local: torch.Tensor, out: torch.Tensor) -> None:
        """Writes the whole vector's sum to ``out`` (one float32) on every rank."""
        if local.numel() != self.local:
            raise ConfigError(f"rank {self.rank} holds {self.local} of the {self.n} values, got {local.numel()}")
        self._shard_sum(local, self.partial)
        if self.world == 1:
            out.copy_(self.partial)
            return
        self.dist.all_gather_into_tensor(self.gathered, self.partial)
        self._tree(self.gathered, out)

    def __call__(self, local: torch.Tensor) -> float:
        out = torch.empty(1, dtype=torch.float32, device=local.device)
        self.into(local, out)
        return float(out.item())


def pairwise(values: torch.Tensor, block: int = DEFAULT_BLOCK) -> float:
    """Halve until a range fits ``block``, sum blocks sequentially, add halves (summation.py:64-85)."""
    v = _checked(values)
    if block < 1:
        raise ConfigError(f"a block of {block} values is not a block")
    out = torch.empty(1, dtype=torch.float32, device=v.device)
    scratch = torch.empty(max(1, scratch_bytes(v.numel(), block)), dtype=torch.uint8, device=v.device)
    pairwise_into(v, out, scratch, block)
    return float(out.item())


def sequential(values: torch.Tensor) -> float:
    """One accumulator from 0.0, left to right (summation.py:56-61)."""
    v = _checked(values)
    out = torch.empty(1, dtype=torch.float32, device=v.device)
    sequential_into(v, out)
    return float(out.item())


def exact(values) -> float:
    """The correctly rounded float64 value of the exact sum of float32 values (tgc's
    summation.exact, summation.py:47-53, which rounds math.fsum's exact running sum once).

    Every finite float32 is a signed integer below 2^24 times 2^(e - 150), with e its biased
    exponent field (1 for subnormals). The integers are read from the bit patterns, summed per
    exponent (as 12-bit halves, so the float64 sums of bincount stay exact below 2^53), and the
    256 sums are combined as one Python integer and rounded once by integer true division. It
    runs with torch on the tensor's own device, so a CUDA tensor is summed where it lies; arrays
    and CPU tensors are summed on the CPU. Non-finite inputs take math.fsum's answer.
    """
    t = values if isinstance(values, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(values))
    t = t.detach().reshape(-1)
    if t.dtype != torch.float32:
        raise ConfigError(f"these orders are about float32, got {t.dtype}")
    if t.numel() == 0:
        raise ConfigError("there is nothing to sum")
    bits = t.contiguous().view(torch.int32)
    field = (bits >> 23) & 0xFF
    if bool((field == 0xFF).any()):
        return math.fsum(t.cpu().double().tolist())
    mant = bits & 0x7FFFFF
    ints = torch.where(field > 0, mant | 0x800000, mant)
    ints = torch.where(bits < 0, -ints, ints)
    slot = field.clamp_min(1).long()
    hi = torch.bincount(slot, weights=(ints >> 12).double(), minlength=256).tolist()
    lo = torch.bincount(slot, weights=(ints & 0xFFF).double(), minlength=256).tolist()
    total = 0
    for k in range(256):
        if hi[k] or lo[k]:
            total += ((int(hi[k]) << 12) + int(lo[k])) << k
    return total / (1 << 150)


def relative_error(approximate: float, reference: float) -> float:
    """|approximate - reference| / |reference| (tgc's summation.relative_error, summation.py:134-139)."""
    if reference == 0.0:
        raise ConfigError("a relative error against zero is undefined")
    return abs(approximate - reference) / abs(reference)
