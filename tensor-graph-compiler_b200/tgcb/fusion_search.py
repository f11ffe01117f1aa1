"""tgc's materialise-or-recompute model, and where the backend's one-pass kernels sit in it.

tgc/schedule/fusion_search.py:36-276 prices a *plan*, a set of values written to memory, on a
DAG of values with a size and a flop count each: every reduction and graph output is written
whatever the plan says, every other value is either written (and read back by each kernel that
needs it) or recomputed inside each kernel that reads it. A plan's cost is its flops, with
work duplicated across kernels counted once per kernel, plus ``MEMORY_WEIGHT`` times its bytes.
``exhaustive`` tries every subset of the interior values; ``materialise_reused`` is the rule
"write anything read twice"; ``cone_dag`` is the shape of the fused cone workload (an
elementwise cone read by several reductions).

This module restates that model with the same semantics, so its plans and costs are tgc's
(tests/golden/models.json holds tgc's own numbers), and adds what the model has no
plan for: the backend lowers reductions that read the same rows into ONE multi-output row
kernel (tgcb/codegen.py), which walks the cone once and reads its inputs once, so the
recomputation the model charges per reduction never happens. ``one_pass`` prices that kernel
with the model's own rules: the kernels rooted at the reductions merge into one, whose
operations are computed once and whose outside inputs are read once. ``dag_of`` flattens a
graph (tgc's or tgcb's) into a ``Dag`` with tgc's per-operation flop costs, so the model can
be run on the real workload graph, and ``predicted_seconds`` turns a plan into time on a
roofline ``Machine`` (tgcb.cost).
"""

from __future__ import annotations

import itertools
from collections.abc import Sequence
from dataclasses import dataclass

from tgcb.errors import ConfigError, ScheduleError

BYTES_PER_ELEMENT = 4
MEMORY_WEIGHT = 10.0


@dataclass(frozen=True)
class Dag:
    """Values in topological order: the values each is computed from, its element count and
    its flops; ``outputs`` and ``barriers`` (reductions) are always written."""

    producers: tuple[tuple[int, ...], ...]
    sizes: tuple[int, ...]
    flops: tuple[int, ...]
    outputs: tuple[int, ...]
    barriers: tuple[int, ...] = ()

    def __post_init__(self) -> None:
        n = len(self.producers)
        if n == 0:
            raise ConfigError("a DAG without values computes nothing")
        if len(self.sizes) != n or len(self.flops) != n:
            raise ConfigError("each value needs exactly one size and one flop count")
        for i, srcs in enumerate(self.producers):
            if any(not 0 <= s < i for s in srcs):
                raise ConfigError(f"value {i} must be computed from earlier values only, got {srcs}")
        if not self.outputs:
            raise ConfigError("a DAG needs at least one output")
        for v in (*self.outputs, *self.barriers):
            if not 0 <= v < n:
                raise ConfigError(f"{v} names no value of this DAG")
            if not self.producers[v]:
                raise ConfigError(f"value {v} is read from memory; it cannot be an output or a reduction")

    @property
    def count(self) -> int:
        return len(self.producers)

    @property
    def leaves(self) -> frozenset[int]:
        return frozenset(i for i, p in enumerate(self.producers) if not p)

    @property
    def required(self) -> frozenset[int]:
        return frozenset(self.outputs) | frozenset(self.barriers)

    @property
    def interior(self) -> tuple[int, ...]:
        """Computed values that no rule forces into memory: the plan's choices."""
        req = self.required
        return tuple(i for i in range(self.count) if self.producers[i] and i not in req)

    def consumers(self, value: int) -> tuple[int, ...]:
        if not 0 <= value < self.count:
            raise ConfigError(f"{value} names no value of this DAG")
        return tuple(i for i, p in enumerate(self.producers) if value in p)

    def fan_out(self, value: int) -> int:
        """Readers of a value, a graph output counting as one more."""
        return len(self.consumers(value)) + (1 if value in self.outputs else 0)


def group_for(dag: Dag, root: int, materialised: frozenset[int]) -> frozenset[int]:
    """The operations of the kernel that writes ``root``: everything upstream of it up to the
    leaves and the other written values."""
    if not dag.producers[root]:
        raise ScheduleError(f"value {root} is read from memory; no kernel computes it")
    seen: set[int] = set()
    stack = [root]
    while stack:
        v = stack.pop()
        if v in seen:
            continue
        seen.add(v)
        stack.extend(s for s in dag.producers[v] if dag.producers[s] and s not in materialised)
    return frozenset(seen)


def normalise(dag: Dag, chosen: Sequence[int]) -> frozenset[int]:
    """A choice plus the values every plan writes."""
    for v in chosen:
        if not 0 <= v < dag.count:
            raise ScheduleError(f"{v} names no value of this DAG")
        if not dag.producers[v]:
            raise ScheduleError(f"value {v} is read from memory already; writing it is no choice")
    return frozenset(chosen) | dag.required


@dataclass
class FusionPlan:
    """A written set, its kernel count, flops and bytes; cost = flops + weight * bytes."""

    materialised: frozenset[int] = frozenset()
    groups: int = 0
    flops: int = 0
    traffic: int = 0
    memory_weight: float = MEMORY_WEIGHT

    @property
    def cost(self) -> float:
        return self.flops + self.traffic * self.memory_weight

    def as_dict(self) -> dict:
        return {"materialised": sorted(self.materialised), "groups": self.groups, "flops": self.flops,
                "traffic": self.traffic, "cost": round(self.cost, 2)}


def groups_of(dag: Dag, chosen: Sequence[int]) -> dict[int, frozenset[int]]:
    written = normalise(dag, chosen)
    return {root: group_for(dag, root, written) for root in sorted(written)}


def _outside_reads(dag: Dag, members: frozenset[int], skip: int | None) -> set[int]:
    """Values a kernel reads from memory: sources of its members that it does not compute."""
    return {s for m in members for s in dag.producers[m] if s not in members and s != skip}


def cost_of(dag: Dag, chosen: Sequence[int], memory_weight: float = MEMORY_WEIGHT) -> FusionPlan:
    """Each written value once, plus each kernel's outside reads once per kernel, plus every
    kernel's flops (an operation in two kernels is paid twice)."""
    if memory_weight < 0:
        raise ConfigError(f"a negative memory weight ({memory_weight}) prices nothing")
    written = normalise(dag, chosen)
    groups = groups_of(dag, chosen)
    flops = sum(dag.flops[m] for members in groups.values() for m in members)
    elements = sum(dag.sizes[v] for v in written)
    for root, members in groups.items():
        elements += sum(dag.sizes[s] for s in _outside_reads(dag, members, root))
    return FusionPlan(written, len(groups), flops, elements * BYTES_PER_ELEMENT, memory_weight)


def times_computed(dag: Dag, chosen: Sequence[int], value: int) -> int:
    if not 0 <= value < dag.count:
        raise ScheduleError(f"{value} names no value of this DAG")
    return sum(1 for members in groups_of(dag, chosen).values() if value in members)


def duplication_factor(dag: Dag, chosen: Sequence[int]) -> float:
    """Operations computed, over distinct operations (1.0: nothing recomputed)."""
    groups = list(groups_of(dag, chosen).values())
    distinct = len(set().union(*groups)) if groups else 0
    if distinct == 0:
        raise ScheduleError("a plan without kernels computes nothing")
    return sum(len(g) for g in groups) / distinct


def materialise_everything(dag: Dag, memory_weight: float = MEMORY_WEIGHT) -> FusionPlan:
    return cost_of(dag, dag.interior, memory_weight)


def materialise_outputs_only(dag: Dag, memory_weight: float = MEMORY_WEIGHT) -> FusionPlan:
    return cost_of(dag, (), memory_weight)


def materialise_reused(dag: Dag, memory_weight: float = MEMORY_WEIGHT) -> FusionPlan:
    """Write every interior value with more than one reader."""
    return cost_of(dag, [v for v in dag.interior if dag.fan_out(v) > 1], memory_weight)


def exhaustive(dag: Dag, memory_weight: float = MEMORY_WEIGHT, limit: int = 16) -> FusionPlan:
    """The cheapest of all 2^interior plans; the first found wins a tie, in order of size."""
    interior = dag.interior
    if len(interior) > limit:
        raise ScheduleError(f"{len(interior)} free values make {2 ** len(interior)} plans; the limit is {limit} values")
    best = materialise_outputs_only(dag, memory_weight)
    for k in range(len(interior) + 1):
        for chosen in itertools.combinations(interior, k):
            plan = cost_of(dag, chosen, memory_weight)
            if plan.cost < best.cost:
                best = plan
    return best


def one_pass(dag: Dag, memory_weight: float = MEMORY_WEIGHT) -> FusionPlan:
    """The backend's plan: only the required values are written, and the kernels rooted at the
    reductions run as ONE kernel (the multi-output row kernel), so each of their operations is
    computed once and each outside input is read once; kernels rooted at the remaining outputs
    are priced as in ``cost_of``."""
    written = dag.required
    groups = groups_of(dag, ())
    fused_roots = [r for r in groups if r in dag.barriers]
    merged = frozenset().union(*(groups[r] for r in fused_roots)) if fused_roots else frozenset()
    others = {r: g for r, g in groups.items() if r not in fused_roots}
    flops = sum(dag.flops[m] for m in merged) + sum(dag.flops[m] for g in others.values() for m in g)
    elements = sum(dag.sizes[v] for v in written)
    elements += sum(dag.sizes[s] for s in _outside_reads(dag, merged, None))
    for root, members in others.items():
        elements += sum(dag.sizes[s] for s in _outside_reads(dag, members, root))
    kernels = (1 if merged else 0) + len(others)
    return FusionPlan(written, kernels, flops, elements * BYTES_PER_ELEMENT, memory_weight)


def chain_dag(length: int = 8, size: int = 4096, intensity: int = 1) -> Dag:
    """``length`` unary operations in a row after one input."""
    if length < 1:
        raise ConfigError(f"a chain needs at least one operation, got {length}")
    if intensity < 1:
        raise ConfigError(f"an intensity below one flop per element ({intensity}) is no work")
    return Dag(producers=((),) + tuple((i,) for i in range(length)), sizes=(size,) * (length + 1),
               flops=(0,) + (size * intensity,) * length, outputs=(length,))


def cone_dag(readers: int = 3, depth: int = 4, size: int = 4096, intensity: int = 1, reduced: int = 64) -> Dag:
    """An input, ``depth`` elementwise operations, ``readers`` reductions of the tip to
    size // reduced values each, and a chain of binary operations joining the reductions."""
    if readers < 2:
        raise ConfigError(f"a cone is read by at least two reductions, got {readers}")
    if depth < 1:
        raise ConfigError(f"a cone has at least one operation, got {depth}")
    if reduced < 1:
        raise ConfigError(f"a reduction factor below one ({reduced}) reduces nothing")
    small = max(size // reduced, 1)
    producers: list[tuple[int, ...]] = [()] + [(i,) for i in range(depth)]
    sizes = [size] * (depth + 1)
    flops = [0] + [size * intensity] * depth
    barriers = []
    for _ in range(readers):
        producers.append((depth,))
        sizes.append(small)
        flops.append(size)
        barriers.append(len(producers) - 1)
    joined = barriers[0]
    for b in barriers[1:]:
        producers.append((joined, b))
        sizes.append(small)
        flops.append(small * intensity)
        joined = len(producers) - 1
    return Dag(tuple(producers), tuple(sizes), tuple(flops), (joined,), tuple(barriers))


def dag_of(graph) -> tuple[Dag, list[str]]:
    """A graph as a Dag (tgc's or tgcb's IR): inputs and constants are read from memory,
    every node's flops are tgc's per-operation cost (tgcb.cost.node_flops), reductions are the
    barriers. Returns the Dag and the value name of each index."""
    from tgcb import cost

    names: list[str] = []
    index: dict[str, int] = {}
    producers, sizes, flops, barriers = [], [], [], []
    for value in graph.inputs:
        index[value.name] = len(names)
        names.append(value.name)
        producers.append(())
        sizes.append(value.shape.elements)
        flops.append(0)
    for node in graph.nodes:
        index[node.name] = len(names)
        names.append(node.name)
        producers.append(tuple(index[i] for i in node.inputs))
        sizes.append(node.output.shape.elements)
        flops.append(int(cost.node_flops(graph, node)))
        if node.op.category == "reduction":
            barriers.append(index[node.name])
    outputs = tuple(index[o] for o in graph.outputs)
    return Dag(tuple(producers), tuple(sizes), tuple(flops), outputs, tuple(barriers)), names


def predicted_seconds(plan: FusionPlan, flops_per_second: float, bytes_per_second: float) -> float:
    """A plan's time on a roofline machine: the larger of its flops and its bytes over the peaks."""
    return max(plan.flops / flops_per_second, plan.traffic / bytes_per_second)


def compare(dag: Dag, memory_weight: float = MEMORY_WEIGHT) -> list[dict]:
    """tgc's three rules and its search, and the backend's one-pass plan, on one DAG."""
    rows = [
        ("everything", materialise_everything(dag, memory_weight)),
        ("outputs only", materialise_outputs_only(dag, memory_weight)),
        ("reused values", materialise_reused(dag, memory_weight)),
        ("exhaustive", exhaustive(dag, memory_weight)),
        ("one pass (tgcb row kernel)", one_pass(dag, memory_weight)),
    ]
    return [{"strategy": name, **plan.as_dict()} for name, plan in rows]
