"""ctypes front end of oracle/bracketing.c. TEST ONLY (see oracle/__init__.py)."""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE = os.path.join(HERE, "bracketing.c")
LIBRARY = os.path.join(HERE, "_build", "libbracketing.so")
CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared"]

_lib = None


def build(force: bool = False) -> str:
    """Compile bracketing.c with gcc (no FMA contraction, no fast-math)."""
    if not force and os.path.exists(LIBRARY) and os.path.getmtime(LIBRARY) >= os.path.getmtime(SOURCE):
        return LIBRARY
    os.makedirs(os.path.dirname(LIBRARY), exist_ok=True)
    tmp = LIBRARY + ".tmp"
    subprocess.run(["gcc", *CFLAGS, SOURCE, "-o", tmp, "-lm"], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIBRARY)
        f = ctypes.c_float
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        lib.oracle_sequential.restype = f
        lib.oracle_sequential.argtypes = [p, i64]
        lib.oracle_pairwise.restype = f
        lib.oracle_pairwise.argtypes = [p, i64, ctypes.c_int]
        lib.oracle_partitioned.restype = f
        lib.oracle_partitioned.argtypes = [p, i64, i64]
        lib.oracle_row_tree.restype = None
        lib.oracle_row_tree.argtypes = [p, i64, i64, ctypes.c_int, ctypes.c_int, p]
        lib.oracle_col_parts.restype = None
        lib.oracle_col_parts.argtypes = [p, i64, i64, i64, ctypes.c_int, p]
        lib.oracle_full_chunks.restype = f
        lib.oracle_full_chunks.argtypes = [p, i64, i64, ctypes.c_int]
        _lib = lib
    return _lib


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def sequential(x) -> float:
    a = _f32(x)
    return float(_load().oracle_sequential(a.ctypes.data, a.size))


def pairwise(x, block: int = 8) -> float:
    a = _f32(x)
    return float(_load().oracle_pairwise(a.ctypes.data, a.size, block))


def partitioned(x, parts: int) -> float:
    a = _f32(x)
    return float(_load().oracle_partitioned(a.ctypes.data, a.size, parts))


def row_tree(x, threads: int, op: str = "sum") -> np.ndarray:
    a = _f32(x)
    rows, cols = a.shape
    out = np.empty(rows, dtype=np.float32)
    _load().oracle_row_tree(a.ctypes.data, rows, cols, threads, 1 if op == "max" else 0, out.ctypes.data)
    return out


def col_parts(x, rows_per_part: int, op: str = "sum") -> np.ndarray:
    a = _f32(x)
    rows, cols = a.shape
    out = np.empty(cols, dtype=np.float32)
    _load().oracle_col_parts(a.ctypes.data, rows, cols, rows_per_part, 1 if op == "max" else 0, out.ctypes.data)
    return out


def full_chunks(x, chunk: int, op: str = "sum") -> float:
    a = _f32(x).reshape(-1)
    return float(_load().oracle_full_chunks(a.ctypes.data, a.size, chunk, 1 if op == "max" else 0))
