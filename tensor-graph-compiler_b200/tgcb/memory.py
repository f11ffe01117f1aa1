"""Execution order, live intervals and the arena plan.

The backend keeps tgc's scheduling and allocation algorithms: a depth-first order from the
outputs (tgc/schedule/order.py:127-155), inclusive live intervals where inputs start before
step 0 and outputs end at the last step (tgc/analysis/liveness.py:70-103), and largest-first
offset assignment against the interference test (tgc/memory/planner.py:128-171).

What changes is what gets a slot. tgc gives every value of the graph a slot because its
generated code materialises every node. The B200 lowering keeps fused intermediates in
registers, so the planner runs over the *kernel steps* and only the values a kernel reads
from or writes to HBM get a slot. Every slot size is rounded up to ``ALIGNMENT`` bytes before
planning, so every offset the largest-first packer produces (a sum of slot ends) is itself a
multiple of ``ALIGNMENT``: 128-bit vector loads and TMA need 16-byte aligned bases and we
keep whole 256-byte lines. Rounding sizes before packing keeps the plan valid by
construction; rounding offsets after packing (tgc/memory/arena.py:124-140) can overlap two
live slots, which tgc itself guards with ``plan_survives_alignment``.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field

from tgcb.errors import AllocationError, ConfigError, ScheduleError

ALIGNMENT = 256


def align_up(offset: int, alignment: int = ALIGNMENT) -> int:
    if alignment <= 0 or alignment & (alignment - 1):
        raise ConfigError(f"an alignment has to be a power of two, got {alignment}")
    if offset < 0:
        raise ConfigError(f"an offset cannot be negative, got {offset}")
    return (offset + alignment - 1) & ~(alignment - 1)


# ----------------------------------------------------------------------------- order


def depth_first_order(graph) -> list:
    """Emit each output's producers depth-first, then anything left (tgc/schedule/order.py:127-155)."""
    done: set[str] = set()
    order: list = []
    producers = {n.name: n for n in graph.nodes}

    # Iterative post-order so a deep chain (a long gradient graph) does not hit the
    # interpreter's recursion limit; visits children in operand order like the recursive form.
    def emit(root) -> None:
        stack = [(root, 0)]
        while stack:
            node, k = stack.pop()
            if node.name in done:
                continue
            if k < len(node.inputs):
                stack.append((node, k + 1))
                parent = producers.get(node.inputs[k])
                if parent is not None and parent.name not in done:
                    stack.append((parent, 0))
                continue
            done.add(node.name)
            order.append(node)

    for name in graph.outputs:
        p = producers.get(name)
        if p is not None:
            emit(p)
    for n in graph.nodes:
        emit(n)
    return order


# ----------------------------------------------------------------------------- liveness


@dataclass
class Interval:
    """Steps [start, end] (inclusive) during which a value must exist (tgc/analysis/liveness.py:24-60)."""

    name: str
    start: int
    end: int
    size: int

    def __post_init__(self) -> None:
        if not self.name:
            raise ConfigError("an interval needs a name")
        if self.end < self.start:
            raise ScheduleError(f"{self.name} ends at {self.end} before it starts at {self.start}")
        if self.size < 0:
            raise ConfigError(f"{self.name} cannot occupy {self.size} bytes")

    def overlaps(self, other: Interval) -> bool:
        return self.start <= other.end and other.start <= self.end


def intervals_for_steps(
    input_names: Sequence[str],
    steps: Sequence[tuple[Sequence[str], Sequence[str]]],
    outputs: Sequence[str],
    sizes: dict[str, int],
) -> list[Interval]:
    """Live intervals over a list of steps, each ``(reads, writes)``.

    The same end rules as tgc's ``compute_intervals``: a graph input starts at -1, a value
    starts at the step that writes it, ends at its last reader, and graph outputs live to
    the last step. Sizes are rounded to ``ALIGNMENT``.
    """
    last = len(steps) - 1
    start: dict[str, int] = {}
    end: dict[str, int] = {}
    for name in input_names:
        start[name] = -1
        end[name] = -1
    for k, (reads, writes) in enumerate(steps):
        for w in writes:
            if w in start and start[w] != -1:
                raise ScheduleError(f"{w} is written by two steps")
            if w not in start:
                start[w] = k
                end[w] = k
        for r in reads:
            if r not in start:
                raise ScheduleError(f"step {k} reads {r} before anything writes it")
            end[r] = max(end[r], k)
    for o in outputs:
        if o in end:
            end[o] = max(last, end[o])
    return [Interval(n, start[n], max(end[n], start[n]), align_up(sizes[n])) for n in start]


def peak_bytes(intervals: Sequence[Interval]) -> int:
    if not intervals:
        return 0
    lo = min(i.start for i in intervals)
    hi = max(i.end for i in intervals)
    return max(sum(i.size for i in intervals if i.start <= s <= i.end) for s in range(lo, hi + 1))


# ----------------------------------------------------------------------------- planner


@dataclass
class Allocation:
    """Bytes [offset, offset+size) of the arena (tgc/memory/planner.py:24-48)."""

    name: str
    offset: int
    size: int

    @property
    def end(self) -> int:
        return self.offset + self.size

    def overlaps(self, other: Allocation) -> bool:
        return self.offset < other.end and other.offset < self.end

    def as_dict(self) -> dict:
        return {"name": self.name, "offset": self.offset, "size": self.size}


@dataclass
class Plan:
    allocations: list[Allocation] = field(default_factory=list)
    strategy: str = ""

    @property
    def arena_bytes(self) -> int:
        return max((a.end for a in self.allocations), default=0)

    def by_name(self) -> dict[str, Allocation]:
        return {a.name: a for a in self.allocations}

    def as_dict(self) -> dict:
        return {"strategy": self.strategy, "tensors": len(self.allocations), "arena_bytes": self.arena_bytes}


def plan_largest_first(intervals: Sequence[Interval]) -> Plan:
    """Biggest first, each at the lowest offset clear of every live neighbour (tgc/memory/planner.py:157-171)."""
    placed: list[tuple[Interval, Allocation]] = []
    for iv in sorted(intervals, key=lambda i: (-i.size, i.start, i.name)):
        blocked = sorted((a for other, a in placed if iv.overlaps(other)), key=lambda a: a.offset)
        offset = 0
        for a in blocked:
            if offset + iv.size <= a.offset:
                break
            offset = max(offset, a.end)
        placed.append((iv, Allocation(iv.name, offset, iv.size)))
    return Plan([a for _, a in placed], "largest first")


def validate_plan(intervals: Sequence[Interval], plan: Plan, alignment: int = ALIGNMENT) -> None:
    """No two simultaneously live values share a byte, and every offset is aligned."""
    where = plan.by_name()
    missing = [i.name for i in intervals if i.name not in where]
    if missing:
        raise AllocationError(f"no placement for {missing}")
    for a in plan.allocations:
        if a.offset % alignment:
            raise AllocationError(f"{a.name} sits at {a.offset}, which is not a multiple of {alignment}")
    for k, first in enumerate(intervals):
        for second in intervals[k + 1 :]:
            if first.overlaps(second) and where[first.name].overlaps(where[second.name]):
                raise AllocationError(
                    f"{first.name} and {second.name} are alive together and share bytes "
                    f"{where[first.name].offset} and {where[second.name].offset}"
                )
