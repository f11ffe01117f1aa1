"""float32 summation orders on the GPU, bit-exact to tgc/analysis/summation.py.

``pairwise`` and ``sequential`` take a 1-D float32 CUDA tensor and return the same Python
float tgc's functions return for the same values (summation.py:56-85), computed by the
library's kernels (tgcb_sum_pairwise_f32, tgcb_sum_sequential_f32). The input checks and
their ``ConfigError`` messages follow tgc's ``_checked`` (summation.py:36-44).
``*_into`` variants write the result to a device scalar on a stream without synchronising.
"""

from __future__ import annotations

import ctypes

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
