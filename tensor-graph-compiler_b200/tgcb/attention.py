"""Streaming attention on the GPU (tgc/analysis/attention.py:97-137).

``streaming_attention(queries, keys, values, block)`` takes float32 CUDA matrices and returns
the same function tgc's version computes, from one fused kernel (``tgcb_streaming_attention_f32``):
one pass over the keys with the running maximum and sum rescaled as blocks arrive, the score
matrix never written to memory. ``block`` is checked as tgc checks it; the kernel's own key
block is 64, which moves rounding, not the result. ``AttentionShape`` mirrors tgc's
(attention.py:44-77).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from tgcb import _lib
from tgcb.errors import ConfigError

WIDTHS = (16, 32, 64, 128)


@dataclass(frozen=True)
class AttentionShape:
    sequence: int
    width: int

    def __post_init__(self) -> None:
        if min(self.sequence, self.width) < 1:
            raise ConfigError(f"a head cannot be {self.sequence} by {self.width}")

    @property
    def input_elements(self) -> int:
        return 3 * self.sequence * self.width

    @property
    def score_elements(self) -> int:
        return self.sequence * self.sequence

    @property
    def arithmetic(self) -> float:
        """Multiply-adds in the two products (attention.py:67-70)."""
        return 4.0 * self.sequence * self.sequence * self.width

    def as_dict(self) -> dict:
        return {"sequence": self.sequence, "width": self.width, "inputs": self.input_elements,
                "scores": self.score_elements}


def streaming_attention_into(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, out: torch.Tensor,
                             stream=None) -> None:
    for name, t in (("queries", queries), ("keys", keys), ("values", values), ("out", out)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32 or t.dim() != 2:
            raise ConfigError(f"{name} must be a float32 CUDA matrix")
        if not t.is_contiguous():
            raise ConfigError(f"{name} must be contiguous")
    sq, width = queries.shape
    sk = keys.shape[0]
    if width not in WIDTHS:
        raise ConfigError(f"the kernel takes widths {WIDTHS}, got {width}")
    if keys.shape[1] != width or values.shape != keys.shape or out.shape != queries.shape:
        raise ConfigError("keys and values must be [keys, width] and out [queries, width]")
    if sq == 0 or sk == 0:
        raise ConfigError("a head needs at least one query and one key")
    _lib.ensure_device(queries.device.index)
    s = stream if stream is not None else torch.cuda.current_stream(queries.device)
    rc = _lib.load().tgcb_streaming_attention_f32(
        ctypes.c_void_p(queries.data_ptr()), ctypes.c_void_p(keys.data_ptr()), ctypes.c_void_p(values.data_ptr()),
        sq, sk, width, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(s.cuda_stream),
    )
    _lib.check(rc, "tgcb_streaming_attention_f32")


def streaming_attention(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, block: int = 128) -> torch.Tensor:
    """softmax(queries keys^T / sqrt(width)) values in one pass over the keys."""
    if block < 1:
        raise ConfigError(f"a block has to hold something, got {block}")
    q, k, v = (t.contiguous() for t in (queries, keys, values))
    out = torch.empty_like(q)
    streaming_attention_into(q, k, v, out)
    return out
