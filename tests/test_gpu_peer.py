"""tgcb_peer_allreduce_avg_f32 on one GPU: a group of one rank (the average is the value
itself), and the bounded wait: a group whose second rank never announces itself makes the
kernel give up after its 4-second budget and record status 5, with the context still usable.
Two real ranks are tested in test_gpu_parallel.py (skipped with fewer than two GPUs)."""

from __future__ import annotations

import ctypes

import pytest
import torch

from tgcb import _lib

pytestmark = pytest.mark.gpu


def _alloc(nbytes):
    lib = _lib.load()
    ptr = ctypes.c_void_p()
    h = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES)()
    _lib.check(lib.tgcb_peer_alloc(nbytes, ctypes.byref(ptr), h), "tgcb_peer_alloc")
    return ptr.value


def _view(ptr, n):
    from tgcb.peer import _DeviceBytes

    return torch.as_tensor(_DeviceBytes(ptr, n * 4), device="cuda:0").view(torch.float32)


def _status(clear=True):
    st = ctypes.c_int(0)
    _lib.check(_lib.load().tgcb_status(1 if clear else 0, ctypes.byref(st)), "tgcb_status")
    return st.value


def _run(desc, segs, slot, epoch, ctas=8):
    arr = (_lib.Segment * len(segs))(*[_lib.Segment(o, c) for o, c in segs])
    return _lib.load().tgcb_peer_allreduce_avg_f32(ctypes.byref(desc), arr, len(segs), slot, epoch, ctas,
                                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_one_rank_group_keeps_its_values(cuda):
    _lib.ensure_device(0)
    n = 1 << 16
    base, flags = _alloc(n * 4), _alloc(_lib.PEER_FLAG_WORDS * 4)
    lib = _lib.load()
    try:
        x = _view(base, n)
        x.copy_(torch.randn(n, generator=torch.Generator().manual_seed(3)).cuda())
        before = x.clone()
        desc = _lib.PeerGroupDesc()
        desc.rank, desc.world, desc.bytes = 0, 1, n * 4
        desc.bases[0], desc.flags[0] = base, flags
        for epoch in (1, 2):  # flags are monotonic: a second call needs no reset
            _lib.check(_run(desc, [(0, 4096), (16 * 4096, n - 4 * 4096)], 0, epoch), "all-reduce")
            torch.cuda.synchronize()
            assert _status() == 0
            assert torch.equal(x, before)
        # slot 0's ready and done words hold the last epoch, its finished count epochs x CTAs
        f = _view(flags, _lib.PEER_FLAG_WORDS).view(torch.int32).cpu()
        assert int(f[0]) == 2 and int(f[4 * _lib.MAX_PEERS]) == 2 and int(f[8 * _lib.MAX_PEERS]) == 2 * 8
    finally:
        torch.cuda.synchronize()
        lib.tgcb_peer_free(ctypes.c_void_p(base))
        lib.tgcb_peer_free(ctypes.c_void_p(flags))


def test_a_rank_that_never_arrives_times_out_with_a_status(cuda):
    _lib.ensure_device(0)
    n = 1024
    base, other, flags, other_flags = _alloc(n * 4), _alloc(n * 4), _alloc(_lib.PEER_FLAG_WORDS * 4), _alloc(
        _lib.PEER_FLAG_WORDS * 4)
    lib = _lib.load()
    try:
        assert _status() == 0
        desc = _lib.PeerGroupDesc()
        desc.rank, desc.world, desc.bytes = 0, 2, n * 4
        desc.bases[0], desc.flags[0] = base, flags
        desc.bases[1], desc.flags[1] = other, other_flags  # nothing runs as rank 1
        _lib.check(_run(desc, [(0, n)], 3, 1, ctas=2), "all-reduce")
        torch.cuda.synchronize()
        assert _status() == 5
        # the context is still usable
        y = torch.ones(16, device="cuda:0") * 2
        assert float(y.sum()) == 32.0
    finally:
        torch.cuda.synchronize()
        for p in (base, other, flags, other_flags):
            lib.tgcb_peer_free(ctypes.c_void_p(p))


def test_bad_arguments_are_refused_before_any_launch(cuda):
    _lib.ensure_device(0)
    desc = _lib.PeerGroupDesc()
    desc.rank, desc.world = 0, 9
    assert _run(desc, [(0, 4)], 0, 1) == _lib.TGCB_E_INVALID
    desc.world = 1
    assert _run(desc, [(0, 4)], 0, 1) == _lib.TGCB_E_INVALID  # null base
    base, flags = _alloc(64), _alloc(_lib.PEER_FLAG_WORDS * 4)
    try:
        desc.bases[0], desc.flags[0] = base, flags
        desc.bytes = 64
        assert _run(desc, [(48, 8)], 0, 1) == _lib.TGCB_E_INVALID  # past the buffer
        assert _run(desc, [(4, 4)], 0, 1) == _lib.TGCB_E_INVALID  # offset not on 16 bytes
        assert _run(desc, [(0, 6)], 0, 1) == _lib.TGCB_E_INVALID  # not a multiple of 4
        assert _run(desc, [(0, 4)], 4, 1) == _lib.TGCB_E_INVALID  # slot
        assert _run(desc, [(0, 4)], 0, 0) == _lib.TGCB_E_INVALID  # epoch 0
        assert _status() == 0
    finally:
        _lib.load().tgcb_peer_free(ctypes.c_void_p(base))
        _lib.load().tgcb_peer_free(ctypes.c_void_p(flags))
