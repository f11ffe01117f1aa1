"""Host-side logic of the peer all-reduce (tgcb/peer.py): how the vectors are shared out and
which tensors a call accepts. The kernel itself is tested on GPUs (test_gpu_peer.py and the
two-rank tests in test_gpu_parallel.py)."""

from __future__ import annotations

import pytest
import torch

from tgcb import _lib, peer
from tgcb.errors import ConfigError


@pytest.mark.parametrize("total,world", [(0, 2), (1, 2), (7, 3), (8, 8), (1049856 // 4, 8), (5, 8)])
def test_shares_cover_every_vector_once_in_rank_order(total, world):
    s = peer.shares(total, world)
    assert len(s) == world
    covered = [i for lo, hi in s for i in range(lo, hi)]
    assert covered == list(range(total))
    sizes = [hi - lo for lo, hi in s]
    assert max(sizes) - min(sizes) <= -(-total // world)


def test_segments_are_offsets_from_the_base():
    buf = torch.zeros(4096, dtype=torch.float32)
    base = buf.data_ptr()
    segs = peer.segments_of([buf[0:1024], buf[2048:2052]], base, buf.numel() * 4)
    assert segs == [(0, 1024), (2048 * 4, 4)]


def test_segments_refuse_what_the_kernel_cannot_take():
    buf = torch.zeros(4096, dtype=torch.float32)
    base, n = buf.data_ptr(), buf.numel() * 4
    with pytest.raises(ConfigError, match="multiple of 4"):
        peer.segments_of([buf[0:6]], base, n)
    with pytest.raises(ConfigError, match="16 bytes"):
        peer.segments_of([buf[1:5]], base, n)
    with pytest.raises(ConfigError, match="outside"):
        peer.segments_of([torch.zeros(8)], base, n)
    with pytest.raises(ConfigError, match="float32"):
        peer.segments_of([buf.view(torch.int32)[0:8]], base, n)
    with pytest.raises(ConfigError, match="overlap"):
        peer.segments_of([buf[0:8], buf[4:12]], base, n)
    with pytest.raises(ConfigError, match="1 to 8"):
        peer.segments_of([buf[4 * i : 4 * i + 4] for i in range(9)], base, n)


def test_the_c_abi_structures_match_the_header():
    import ctypes

    assert ctypes.sizeof(_lib.PeerGroupDesc) == 8 + 2 * 8 * _lib.MAX_PEERS + 8
    assert ctypes.sizeof(_lib.Segment) == 16
    import os

    header = open(os.path.join(os.path.dirname(__file__), "..", "include", "tgcb.h")).read()
    assert f"#define TGCB_MAX_PEERS {_lib.MAX_PEERS}" in header
    assert f"#define TGCB_PEER_HANDLE_BYTES {_lib.PEER_HANDLE_BYTES}" in header
    assert "#define TGCB_PEER_FLAG_WORDS (2 * TGCB_PEER_SLOTS * TGCB_MAX_PEERS + TGCB_PEER_SLOTS)" in header
    assert _lib.PEER_FLAG_WORDS == 2 * 4 * _lib.MAX_PEERS + 4
    assert "#define TGCB_PEER_SLOTS 4" in header and peer.SLOTS == 4
