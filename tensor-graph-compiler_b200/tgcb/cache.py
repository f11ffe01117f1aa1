"""Compiled graphs kept by shape signature, so repeated shapes skip lowering and loading.

tgc keys compiled artefacts by ``shape_signature`` (tgc/runtime/cache.py:57-66): the graph's
structural hash (tgc/ir/isomorphism.py:52-95: a bottom-up blake2b tree hash over operations,
attributes, dtypes and input positions, commutative operands sorted, taken over the outputs)
plus the input shapes. tgc only simulates the cache's eviction policies
(cache.py:100-166); here ``PlanCache`` holds real ``CompiledGraph`` objects (their loaded
module, launch plan and device arena) with the same policies, and can write each entry's
graph in tgc's text format (``tgcb.serialize``) to a directory so a new process can compile
them again ahead of use (``warm``); the NVRTC cubins themselves are cached on disk by content
hash, so that recompilation is a lookup.
"""

from __future__ import annotations

import hashlib
import os
import random
import time
from collections.abc import Callable
from dataclasses import dataclass

from tgcb import serialize
from tgcb.errors import ConfigError, GraphError

DIGEST_BITS = 64
POLICIES = ("least recently used", "least frequently used", "first in", "random")


def _digest(text: str) -> str:
    return hashlib.blake2b(text.encode(), digest_size=DIGEST_BITS // 8).hexdigest()


def _attrs_text(node) -> str:
    return ",".join(f"{k}={v}" for k, v in sorted(node.attrs.items()))


def node_identities(graph) -> dict[str, str]:
    """Name-independent identity of every value (isomorphism.py:66-86): inputs by position,
    dtype and shape; a node by its operation, attributes, dtype and its inputs' identities."""
    ids: dict[str, str] = {}
    for index, value in enumerate(graph.inputs):
        ids[value.name] = _digest(f"input:{index}:{value.dtype.name}:{value.shape}")
    for node in graph.nodes:
        parts = [ids[n] for n in node.inputs]
        if node.op.commutative:
            parts.sort()
        ids[node.name] = _digest(f"{node.op.name}|{_attrs_text(node)}|{node.output.dtype.name}|{'.'.join(parts)}")
    return ids


def structural_hash(graph) -> str:
    """One hash over the graph's outputs in order (isomorphism.py:89-95)."""
    ids = node_identities(graph)
    missing = [n for n in graph.outputs if n not in ids]
    if missing:
        raise GraphError(f"{missing} are outputs with no identity")
    return _digest("|".join(ids[n] for n in graph.outputs))


def shape_signature(graph) -> str:
    """Structure plus input shapes (cache.py:57-66): every arena offset and tile count in a
    compiled plan is a number, so the shapes are part of the key."""
    return f"{structural_hash(graph)}:{';'.join(str(v.shape) for v in graph.inputs)}"


@dataclass
class CacheStats:
    hits: int = 0
    misses: int = 0
    evictions: int = 0
    compile_seconds: float = 0.0

    @property
    def requests(self) -> int:
        return self.hits + self.misses

    @property
    def hit_rate(self) -> float:
        return self.hits / self.requests if self.requests else 0.0

    def as_dict(self) -> dict:
        return {"requests": self.requests, "hits": self.hits, "misses": self.misses, "evictions": self.evictions,
                "hit_rate": round(self.hit_rate, 4), "compile_seconds": round(self.compile_seconds, 3)}


class PlanCache:
    """At most ``capacity`` compiled graphs, keyed by (shape signature, device).

    ``compile`` defaults to ``tgcb.runtime.compile_graph``; a miss into a full cache drops the
    entry ``policy`` picks (cache.py:100-117; Belady's "optimal" needs the future and is left to
    tgc's simulator). With ``directory`` every compiled graph is also written there as
    ``<signature digest>.tgc``.
    """

    def __init__(self, capacity: int = 16, policy: str = "least recently used", *, directory: str | None = None,
                 compile: Callable | None = None, seed: int = 0):
        if capacity < 1:
            raise ConfigError(f"a cache has to hold something, got {capacity}")
        if policy not in POLICIES:
            raise ConfigError(f"unknown policy {policy!r}, expected one of {list(POLICIES)}")
        self.capacity, self.policy, self.directory = capacity, policy, directory
        self._compile = compile
        self._rng = random.Random(seed)
        self._entries: dict[tuple[str, int | None], object] = {}
        self._order: list[tuple[str, int | None]] = []  # insertion order, for "first in"
        self._used_at: dict[tuple[str, int | None], int] = {}
        self._seen: dict[tuple[str, int | None], int] = {}
        self._clock = 0
        self.stats = CacheStats()

    def __len__(self) -> int:
        return len(self._entries)

    def __contains__(self, graph) -> bool:
        return any(k[0] == shape_signature(graph) for k in self._entries)

    def keys(self) -> list[tuple[str, int | None]]:
        return list(self._order)

    def _victim(self) -> tuple[str, int | None]:
        held = self._order
        if self.policy == "least recently used":
            return min(held, key=lambda k: self._used_at[k])
        if self.policy == "least frequently used":
            return min(held, key=lambda k: (self._seen[k], self._used_at[k]))
        if self.policy == "first in":
            return held[0]
        return self._rng.choice(held)

    def get(self, graph, *, device: int | None = None, **compile_kwargs):
        """The compiled graph for ``graph``'s structure and shapes, compiling it on a miss."""
        key = (shape_signature(graph), device)
        self._clock += 1
        self._seen[key] = self._seen.get(key, 0) + 1
        if key in self._entries:
            self.stats.hits += 1
            self._used_at[key] = self._clock
            return self._entries[key]
        self.stats.misses += 1
        compile_fn = self._compile
        if compile_fn is None:
            from tgcb.runtime import compile_graph as compile_fn
        t0 = time.perf_counter()
        compiled = compile_fn(graph, device=device, **compile_kwargs) if device is not None else compile_fn(graph, **compile_kwargs)
        self.stats.compile_seconds += time.perf_counter() - t0
        if len(self._entries) >= self.capacity:
            victim = self._victim()
            self._order.remove(victim)
            del self._entries[victim]
            self.stats.evictions += 1
        self._entries[key] = compiled
        self._order.append(key)
        self._used_at[key] = self._clock
        if self.directory:
            os.makedirs(self.directory, exist_ok=True)
            path = os.path.join(self.directory, f"{_digest(key[0])}.tgc")
            if not os.path.exists(path):
                with open(path, "w") as f:
                    f.write(serialize.dumps(graph))
        return compiled

    def warm(self, *, device: int | None = None, limit: int | None = None) -> int:
        """Compile the graphs saved in ``directory`` (up to ``capacity`` or ``limit``); returns how many."""
        if not self.directory or not os.path.isdir(self.directory):
            return 0
        names = sorted(n for n in os.listdir(self.directory) if n.endswith(".tgc"))
        count = 0
        for name in names[: min(self.capacity, limit or self.capacity)]:
            with open(os.path.join(self.directory, name)) as f:
                self.get(serialize.loads(f.read()), device=device)
            count += 1
        return count

    def clear(self) -> None:
        self._entries.clear()
        self._order.clear()
        self._used_at.clear()
        self._seen.clear()
