"""tgc's all-reduce model, printed beside the NCCL all-reduce the backend really runs.

tgc has no transport: tgc/parallel/collective.py:44-379 prices a gradient all-reduce with a
link (bandwidth and start-up latency) and two algorithms, and models bucketing and the overlap
with the backward pass. Here the training step averages its gradients with NCCL over NVLink
(tgcb.parallel); this module restates the model so each measured all-reduce can be reported
next to the time the model predicts for it, on a link whose numbers come from measurement
(``nvlink``) instead of tgc's ``FAST``/``SLOW`` placeholders.

The formulas are tgc's (they are what is being compared against): a ring reduction is
2(n - 1) messages of size/n each, a halving tree 2 ceil(log2 n) messages of the whole tensor;
per-device ring volume 2 size (n - 1)/n; buckets concatenate tensors until the next one would
overflow; ``exposed_time`` releases one layer's gradients per equal slice of the backward pass
and runs each layer's reduction as soon as both it and the previous reduction are done.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from dataclasses import dataclass

from tgcb.errors import ConfigError

BYTES_PER_ELEMENT = 4


@dataclass
class Link:
    """A connection between devices: bytes per second and a start-up latency per message."""

    name: str
    bytes_per_second: float
    latency_seconds: float

    def __post_init__(self) -> None:
        if self.bytes_per_second <= 0:
            raise ConfigError("a link's bandwidth must be positive")
        if self.latency_seconds < 0:
            raise ConfigError("a link's latency cannot be negative")

    def time_for(self, moved: float) -> float:
        if moved < 0:
            raise ConfigError(f"a message of {moved} bytes is not a message")
        return self.latency_seconds + moved / self.bytes_per_second

    def as_dict(self) -> dict:
        return {"link": self.name, "bytes_per_second": self.bytes_per_second, "latency_seconds": self.latency_seconds}


FAST = Link("fast", 2.0e11, 2e-6)  # tgc's placeholders
SLOW = Link("slow", 1.2e10, 1e-5)

# B200 NVLink 5 through NVSwitch: a peer copy measured 770 GB/s per direction on this machine
# type; the start-up latency is the caller's measurement (a one-float all-reduce), if it has one.
NVLINK_PEER_COPY_BYTES_PER_SECOND = 770e9


def nvlink(latency_seconds: float = 2e-6, bytes_per_second: float = NVLINK_PEER_COPY_BYTES_PER_SECOND) -> Link:
    return Link("nvlink5", bytes_per_second, latency_seconds)


def _check(size_bytes: float, devices: int) -> None:
    if size_bytes < 0:
        raise ConfigError(f"a tensor of {size_bytes} bytes is not a tensor")
    if devices < 1:
        raise ConfigError(f"an all-reduce needs at least one device, got {devices}")


def ring_time(size_bytes: float, devices: int, link: Link = FAST) -> float:
    _check(size_bytes, devices)
    if devices == 1:
        return 0.0
    return 2 * (devices - 1) * link.time_for(size_bytes / devices)


def tree_time(size_bytes: float, devices: int, link: Link = FAST) -> float:
    _check(size_bytes, devices)
    if devices == 1:
        return 0.0
    return 2 * math.ceil(math.log2(devices)) * link.time_for(size_bytes)


def ring_volume(size_bytes: float, devices: int) -> float:
    """Bytes each device sends in a ring all-reduce: no correct method sends fewer."""
    _check(size_bytes, devices)
    return 0.0 if devices == 1 else 2.0 * size_bytes * (devices - 1) / devices


def tree_volume(size_bytes: float, devices: int) -> float:
    _check(size_bytes, devices)
    return 0.0 if devices == 1 else 2.0 * size_bytes * math.ceil(math.log2(devices))


def bus_bandwidth(size_bytes: float, devices: int, seconds: float) -> float:
    """NCCL's bus bandwidth of an all-reduce: the ring volume per device over the time."""
    if seconds <= 0:
        raise ConfigError("a measured time must be positive")
    return ring_volume(size_bytes, devices) / seconds


def bucket_time(tensors: Sequence[int], devices: int, link: Link = FAST, bucket_bytes: int = 0) -> float:
    """Ring time of many tensors, one reduction each (bucket_bytes 0) or concatenated into
    buckets that are closed before the tensor that would overflow them."""
    if not tensors:
        raise ConfigError("there are no tensors to reduce")
    if bucket_bytes < 0:
        raise ConfigError(f"a bucket of {bucket_bytes} bytes is not a bucket")
    if bucket_bytes == 0:
        return sum(ring_time(t, devices, link) for t in tensors)
    total, current = 0.0, 0
    for t in tensors:
        if current and current + t > bucket_bytes:
            total += ring_time(current, devices, link)
            current = 0
        current += t
    return total + (ring_time(current, devices, link) if current else 0.0)


def gradient_sizes(layers: int = 48, width: int = 1024) -> list[int]:
    """One width x width matrix and two width vectors per layer, in bytes."""
    if min(layers, width) < 1:
        raise ConfigError("a model needs at least one layer of positive width")
    return [s for _ in range(layers) for s in (width * width * BYTES_PER_ELEMENT, width * BYTES_PER_ELEMENT,
                                               width * BYTES_PER_ELEMENT)]


def exposed_time(layers: int = 48, width: int = 1024, devices: int = 8, link: Link = FAST,
                 backward_seconds: float = 0.05, sizes: Sequence[int] | None = None) -> dict:
    """Communication left after the backward pass: layer i's gradients are released at
    (i + 1)/layers of the backward pass and reduced as one ring after both the release and
    the previous reduction. ``sizes`` (bytes, grouped ``len(sizes) // layers`` per layer)
    replaces tgc's synthetic stack when given, so the model can price a real gradient set."""
    if backward_seconds <= 0:
        raise ConfigError(f"a backward pass takes time, not {backward_seconds} s")
    sizes = list(sizes) if sizes is not None else gradient_sizes(layers, width)
    per_layer = len(sizes) // layers
    if per_layer < 1:
        raise ConfigError(f"{len(sizes)} gradients do not fill {layers} layers")
    slot = backward_seconds / layers
    done = 0.0
    for i in range(layers):
        chunk = sum(sizes[i * per_layer:(i + 1) * per_layer])
        done = max(slot * (i + 1), done) + ring_time(chunk, devices, link)
    last = sum(sizes[(layers - 1) * per_layer:])
    serial = bucket_time(sizes, devices, link, bucket_bytes=1 << 24)
    exposed = max(done - backward_seconds, 0.0)
    return {
        "backward_seconds": backward_seconds,
        "communication_seconds": serial,
        "exposed_seconds": exposed,
        "floor_seconds": ring_time(last, devices, link),
        "hidden_share": round(1.0 - exposed / serial, 4) if serial else 0.0,
        "exposed_share_of_the_step": round(exposed / backward_seconds, 6),
    }
