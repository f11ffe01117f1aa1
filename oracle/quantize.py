"""Restatement of tgc's symmetric per-row int8 quantisation. TEST ONLY.

tgc/analysis/quantize.py:90-99 (symmetric_scheme): largest = float(|row|.max()) as a Python
double; scale = largest / 127 (Scheme(bits=8).high = 127), or 1.0 for an all-zero row.
quantize.py:125-128 (quantise): (values - 0.0) / scale, round half to even, clamp to
[-128, 127]; torch divides the float32 tensor by the Python-double scale in float32, i.e. by
float32(scale), which tests/test_oracle.py pins against tgc's own quantise on the golden
matrices. per_row_schemes (quantize.py:229-233) applies it to each row.
"""

from __future__ import annotations

import numpy as np


def row_scales(values: np.ndarray) -> np.ndarray:
    """float32 scale per row: float32(double(max|row|) / 127), 1.0 for a zero row."""
    v = np.asarray(values, dtype=np.float32)
    largest = np.abs(v).max(axis=1).astype(np.float64)
    scale = largest / 127.0
    scale[largest == 0.0] = 1.0
    return scale.astype(np.float32)


def quantise_rows(values: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(q int8 [rows, cols], scale float32 [rows])."""
    v = np.asarray(values, dtype=np.float32)
    s = row_scales(v)
    scaled = (v / s[:, None]).astype(np.float32)
    q = np.clip(np.rint(scaled), -128, 127).astype(np.int8)
    return q, s


def dequantise_rows(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """quantize.py:131-133: integers * scale + 0.0, in float32."""
    return (q.astype(np.float32) * scale[:, None].astype(np.float32)).astype(np.float32)


def int_matmul(qa: np.ndarray, qb: np.ndarray) -> np.ndarray:
    """Exact int32 product of int8 matrices [M,K] @ [K,N].

    Every partial sum is an integer of magnitude <= K*128*128, far below 2**53 for any K this
    backend tiles, so a float64 GEMM computes each dot product exactly; the result equals
    tgc's interpreter's int32 ``matmul`` of the int32 casts (reference.py:86-87).
    """
    k = qa.shape[1]
    if k * 128 * 128 >= 2**53:
        raise ValueError("contraction too long for an exact float64 product")
    return (qa.astype(np.float64) @ qb.astype(np.float64)).astype(np.int32)
