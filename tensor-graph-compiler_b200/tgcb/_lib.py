"""ctypes binding of libtgcb.so (declared in include/tgcb.h).

There is no fallback: if the library is missing the import of anything that launches work
raises, naming the build command. Statuses map onto tgc's exception classes:
TGCB_E_INVALID -> AllocationError/ConfigError, TGCB_E_COMPILE -> CodegenError,
TGCB_E_CUDA / TGCB_E_DEVICE -> DeviceError.
"""

from __future__ import annotations

import ctypes
import os
import threading

from tgcb.errors import AllocationError, CodegenError, ConfigError, DeviceError

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(PACKAGE_DIR, "libtgcb.so")

TGCB_OK = 0
TGCB_E_INVALID = -1
TGCB_E_CUDA = -2
TGCB_E_COMPILE = -3
TGCB_E_DEVICE = -4
TGCB_E_NOT_FOUND = -5
MAX_INPUTS = 48


class OperandDesc(ctypes.Structure):
    _fields_ = [
        ("input_index", ctypes.c_int32),
        ("elem_bytes", ctypes.c_uint32),
        ("arena_offset", ctypes.c_uint64),
        ("rows", ctypes.c_uint64),
        ("cols", ctypes.c_uint64),
        ("box_cols", ctypes.c_uint32),
        ("box_rows", ctypes.c_uint32),
        ("swizzle", ctypes.c_uint32),
        ("chunks", ctypes.c_uint32),
    ]


class LaunchDesc(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_char * 96),
        ("grid", ctypes.c_uint32 * 3),
        ("block", ctypes.c_uint32 * 3),
        ("smem_bytes", ctypes.c_uint32),
        ("is_gemm", ctypes.c_uint32),
        ("a", OperandDesc),
        ("b", OperandDesc),
        ("a2", OperandDesc),
        ("b2", OperandDesc),
        ("counter_offset", ctypes.c_uint64),
        ("counter_bytes", ctypes.c_uint64),
    ]


# Every symbol include/tgcb.h declares, with its ctypes signature.
MAX_PEERS = 8
PEER_HANDLE_BYTES = 64
PEER_FLAG_WORDS = 2 * 4 * MAX_PEERS + 4


class PeerGroupDesc(ctypes.Structure):
    """tgcb_peer_group: one rank's view of every rank's base address and flag words."""

    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("bases", ctypes.c_void_p * MAX_PEERS),
        ("flags", ctypes.c_void_p * MAX_PEERS),
        ("bytes", ctypes.c_uint64),
    ]


class Segment(ctypes.Structure):
    """tgcb_segment: float32 values at a byte offset from every rank's base."""

    _fields_ = [("offset", ctypes.c_uint64), ("count", ctypes.c_uint64)]


SIGNATURES = {
    "tgcb_version": (ctypes.c_char_p, []),
    "tgcb_last_error": (ctypes.c_char_p, []),
    "tgcb_init": (ctypes.c_int, [ctypes.c_int]),
    "tgcb_device_count": (ctypes.c_int, []),
    "tgcb_compile_cubin": (
        ctypes.c_int,
        [
            ctypes.c_char_p,
            ctypes.c_char_p,
            ctypes.POINTER(ctypes.c_char_p),
            ctypes.c_int,
            ctypes.POINTER(ctypes.c_void_p),
            ctypes.POINTER(ctypes.c_size_t),
            ctypes.POINTER(ctypes.c_void_p),
        ],
    ),
    "tgcb_free": (None, [ctypes.c_void_p]),
    "tgcb_module_load": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "tgcb_module_unload": (ctypes.c_int, [ctypes.c_void_p]),
    "tgcb_plan_create": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.POINTER(LaunchDesc), ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)],
    ),
    "tgcb_plan_destroy": (None, [ctypes.c_void_p]),
    "tgcb_plan_set_input_count": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "tgcb_plan_run": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_void_p],
    ),
    "tgcb_plan_launch_count": (ctypes.c_int, [ctypes.c_void_p]),
    "tgcb_plan_run_profiled": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)],
    ),
    "tgcb_delay": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p]),
    "tgcb_plan_run_range": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_void_p],
    ),
    "tgcb_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "tgcb_sum_pairwise_scratch_bytes": (ctypes.c_size_t, [ctypes.c_uint64, ctypes.c_int]),
    "tgcb_sum_pairwise_f32": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
    ),
    "tgcb_sum_sequential_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]),
    "tgcb_sum_perfect_tree_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]),
    "tgcb_streaming_attention_f32": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
         ctypes.c_void_p, ctypes.c_void_p],
    ),
    "tgcb_sum_pairwise_f32_noalloc": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "tgcb_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "tgcb_peer_free": (ctypes.c_int, [ctypes.c_void_p]),
    "tgcb_peer_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "tgcb_peer_close": (ctypes.c_int, [ctypes.c_void_p]),
    "tgcb_peer_allreduce_avg_f32": (
        ctypes.c_int,
        [ctypes.POINTER(PeerGroupDesc), ctypes.POINTER(Segment), ctypes.c_int, ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
         ctypes.c_void_p],
    ),
    "tgcb_quantise_rows_i8": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
}

_lib = None
_lock = threading.Lock()
_initialised: set[int] = set()


def load() -> ctypes.CDLL:
    """Load libtgcb.so from the package directory; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIBRARY):
            raise DeviceError(
                f"{LIBRARY} is missing: build it with `python -m tgcb._build` "
                "(or __graft_entry__.build()); the backend has no fallback"
            )
        lib = ctypes.CDLL(LIBRARY)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return (load().tgcb_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == TGCB_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == TGCB_E_INVALID:
        raise AllocationError(msg)
    if rc == TGCB_E_COMPILE:
        raise CodegenError(msg)
    if rc == TGCB_E_NOT_FOUND:
        raise ConfigError(msg)
    raise DeviceError(msg)


def ensure_device(device: int) -> None:
    if device in _initialised:
        return
    check(load().tgcb_init(device), f"tgcb_init({device})")
    _initialised.add(device)
