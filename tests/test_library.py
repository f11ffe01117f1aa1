"""The C-ABI library loads on a host without a GPU and exports every declared entry point."""

from __future__ import annotations

import ctypes
import os
import re

import pytest
from conftest import REPO

from tgcb import _lib


def declared_functions() -> list[str]:
    with open(os.path.join(REPO, "include", "tgcb.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tgcb_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(_lib.SIGNATURES)


def test_version_and_device_count():
    lib = _lib.load()
    assert lib.tgcb_version().startswith(b"tgcb")
    import torch

    if not torch.cuda.is_available():
        assert lib.tgcb_device_count() == 0


def test_argument_errors_need_no_gpu():
    lib = _lib.load()
    assert lib.tgcb_sum_pairwise_f32(None, 10, 8, None, None, 0, None) == _lib.TGCB_E_INVALID
    assert "null" in _lib.last_error()
    assert lib.tgcb_plan_run(None, None, None, 0, None) == _lib.TGCB_E_INVALID
    assert lib.tgcb_plan_set_input_count(None, 1) == _lib.TGCB_E_INVALID
    assert lib.tgcb_quantise_rows_i8(None, 0, 0, None, None, None) == _lib.TGCB_E_INVALID
    assert lib.tgcb_sum_pairwise_scratch_bytes(1 << 26, 8) > 0


def test_compile_reports_nvrtc_log():
    lib = _lib.load()
    blob, size, log = ctypes.c_void_p(), ctypes.c_size_t(), ctypes.c_void_p()
    rc = lib.tgcb_compile_cubin(b"int x = ;", None, None, 0, ctypes.byref(blob), ctypes.byref(size), ctypes.byref(log))
    assert rc == _lib.TGCB_E_COMPILE
    assert log.value
    assert b"error" in ctypes.string_at(log.value)
    lib.tgcb_free(log)


def test_no_cpu_fallback():
    import torch

    from tgcb import ir, runtime, workloads
    from tgcb.errors import DeviceError

    if torch.cuda.is_available():
        pytest.skip("this checks the behaviour without a GPU")
    with pytest.raises(DeviceError):
        runtime.compile_graph(workloads.cone_graph(ir.Builder, rows=8, cols=8))
