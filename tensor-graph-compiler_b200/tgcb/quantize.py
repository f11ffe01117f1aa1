"""Per-row symmetric int8 quantisation on the GPU, bit-exact to tgc/analysis/quantize.py.

``quantise_rows(values)`` returns what ``per_row_schemes(values, 8)`` followed by
``quantise(row, scheme)`` for every row gives in tgc (quantize.py:90-128, 229-233): the
integers as an int8 tensor and each row's scale as float32 (the value torch divides by).
Dequantisation is not here: it is part of the graph (cast, then a multiply per scale
vector) so it runs fused into the int8 GEMM's epilogue. Error behaviour follows tgc:
``ConfigError`` for an empty input or a non-matrix.
"""

from __future__ import annotations

import ctypes

import torch

from tgcb import _lib
from tgcb.errors import ConfigError


def quantise_rows_into(values: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, stream=None) -> None:
    rows, cols = values.shape
    _lib.ensure_device(values.device.index)
    s = stream if stream is not None else torch.cuda.current_stream(values.device)
    rc = _lib.load().tgcb_quantise_rows_i8(
        ctypes.c_void_p(values.data_ptr()), rows, cols, ctypes.c_void_p(q.data_ptr()),
        ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(s.cuda_stream),
    )
    _lib.check(rc, "tgcb_quantise_rows_i8")


def quantise_rows(values: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    if not isinstance(values, torch.Tensor) or not values.is_cuda:
        raise ConfigError("quantise_rows takes a CUDA tensor")
    if values.dim() != 2:
        raise ConfigError(f"per row schemes need a matrix, got rank {values.dim()}")
    if values.numel() == 0:
        raise ConfigError("there is nothing to quantise")
    v = values.to(torch.float32).contiguous()
    q = torch.empty(v.shape, dtype=torch.int8, device=v.device)
    scale = torch.empty(v.shape[0], dtype=torch.float32, device=v.device)
    quantise_rows_into(v, q, scale)
    return q, scale
