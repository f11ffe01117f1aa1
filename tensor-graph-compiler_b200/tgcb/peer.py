"""Device memory shared by the ranks of one box over NVLink, and the all-reduce that runs on it.

tgc prices the all-reduce of data-parallel gradients with a ring model and never moves a byte
(tgc/parallel/collective.py:76-113). ``PeerGroup`` gives every rank (one process per GPU) a
buffer that all ranks of the box can read and write: it is allocated and exported by
``tgcb_peer_alloc`` on each rank, the 64-byte IPC handles are exchanged through the process
group (``all_gather_object``), and each rank maps the others' buffers with ``tgcb_peer_open``
(plain peer mappings over NVLink/NVSwitch, no multicast). A compiled graph whose arena is this
buffer (``PeerGroup.buffer``) has its outputs at the same offsets on every rank, so
``allreduce_avg`` can average them in place with one kernel per rank
(``tgcb_peer_allreduce_avg_f32``): rank r sums share r of the values over the ranks in rank
order and stores the result on every rank, so the averages are bit-identical on all ranks and
on every run. A call's waits for other ranks are bounded; a rank that gives up records a status
that ``CompiledGraph.check_status`` raises as ``DeviceError``.
"""

from __future__ import annotations

import ctypes

from tgcb import _lib
from tgcb.errors import ConfigError

SLOTS = 4


def shares(total_vectors: int, world: int) -> list[tuple[int, int]]:
    """[first, end) of the 16-byte vectors each rank owns, as the kernel splits them."""
    share = -(-total_vectors // world)
    return [(min(r * share, total_vectors), min((r + 1) * share, total_vectors)) for r in range(world)]


def segments_of(tensors, base: int, nbytes: int) -> list[tuple[int, int]]:
    """(byte offset from ``base``, float count) of each float32 tensor; each must be contiguous,
    lie inside the ``nbytes`` buffer at ``base``, start on 16 bytes and hold a multiple of 4."""
    segs = []
    for t in tensors:
        if str(t.dtype) != "torch.float32" or not t.is_contiguous():
            raise ConfigError("peer all-reduce takes contiguous float32 tensors")
        off = t.data_ptr() - base
        size = t.numel() * 4
        if off < 0 or off + size > nbytes:
            raise ConfigError("a tensor to all-reduce lies outside the peer buffer")
        if off % 16 or t.numel() % 4 or t.numel() == 0:
            raise ConfigError("peer all-reduce segments start on 16 bytes and hold a positive multiple of 4 floats")
        segs.append((off, t.numel()))
    if not 1 <= len(segs) <= 8:
        raise ConfigError("peer all-reduce takes 1 to 8 tensors per call")
    spans = sorted((o, o + 4 * c) for o, c in segs)
    if any(a[1] > b[0] for a, b in zip(spans, spans[1:])):
        raise ConfigError("tensors to all-reduce in one call must not overlap (each element would be averaged twice)")
    return segs


class _DeviceBytes:
    """``__cuda_array_interface__`` over memory this module owns, so torch can view it."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerGroup:
    """One ``nbytes`` buffer per rank, mapped into every rank of the process group, plus flag
    words. Every rank must construct it (it exchanges handles collectively) and ``close`` it."""

    def __init__(self, dist, nbytes: int, device: int, group=None):
        import torch

        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_PEERS:
            raise ConfigError(f"a peer group has at most {_lib.MAX_PEERS} ranks, got {self.world}")
        lib = _lib.load()
        _lib.ensure_device(device)
        self.device = device
        self.nbytes = nbytes
        self._own: list[int] = []
        self._opened: list[int] = []
        handles = []
        with torch.cuda.device(device):
            for size in (nbytes, _lib.PEER_FLAG_WORDS * 4):
                ptr = ctypes.c_void_p()
                h = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES)()
                _lib.check(lib.tgcb_peer_alloc(size, ctypes.byref(ptr), h), "allocating a peer buffer")
                self._own.append(ptr.value)
                handles.append(bytes(h))
            gathered = [None] * self.world
            dist.all_gather_object(gathered, tuple(handles), group=group)
            desc = _lib.PeerGroupDesc()
            desc.rank, desc.world, desc.bytes = self.rank, self.world, nbytes
            for r, (hb, hf) in enumerate(gathered):
                if r == self.rank:
                    desc.bases[r], desc.flags[r] = self._own
                    continue
                mapped = []
                for hbytes in (hb, hf):
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.tgcb_peer_open((ctypes.c_ubyte * len(hbytes)).from_buffer_copy(hbytes), ctypes.byref(ptr)),
                               f"mapping rank {r}'s peer buffer")
                    self._opened.append(ptr.value)
                    mapped.append(ptr.value)
                desc.bases[r], desc.flags[r] = mapped
        self.desc = desc
        self.buffer = torch.as_tensor(_DeviceBytes(self._own[0], nbytes), device=f"cuda:{device}")
        self.epochs = [0] * SLOTS

    def allreduce_avg(self, tensors, slot: int, stream, ctas: int) -> None:
        """Average ``tensors`` (views of ``buffer`` at the same offsets on every rank) over the
        ranks in place, as one kernel of ``ctas`` CTAs queued on ``stream``. Every rank makes
        the same calls with the same arguments in the same order per slot."""
        if not 0 <= slot < SLOTS:
            raise ConfigError(f"slot {slot} is outside 0..{SLOTS - 1}")
        segs = segments_of(tensors, self._own[0], self.nbytes)
        arr = (_lib.Segment * len(segs))(*[_lib.Segment(o, c) for o, c in segs])
        self.epochs[slot] += 1
        rc = _lib.load().tgcb_peer_allreduce_avg_f32(ctypes.byref(self.desc), arr, len(segs), slot, self.epochs[slot], ctas,
                                                     ctypes.c_void_p(stream.cuda_stream))
        _lib.check(rc, "peer all-reduce")

    def close(self) -> None:
        """Unmap the other ranks' buffers and free this rank's, after every rank has finished
        using them (a barrier of the process group)."""
        import torch

        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        self.dist.barrier(group=self.group)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.check(lib.tgcb_peer_close(ctypes.c_void_p(p)), "unmapping a peer buffer")
            self._opened = []
            self.dist.barrier(group=self.group)
            for p in self._own:
                _lib.check(lib.tgcb_peer_free(ctypes.c_void_p(p)), "freeing a peer buffer")
        self._own = []
