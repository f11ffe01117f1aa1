"""Roofline predictions for graphs, with a B200 entry made from measured peaks.

tgc's cost model (tgc/analysis/cost.py:27-181) is a roofline: a graph's arithmetic over a
machine's arithmetic peak against the bytes it moves over the bandwidth, the larger of the two
being the prediction. Its machines are placeholders (``GPU`` is 20 TFLOP/s and 1.5 TB/s,
cost.py:58). This module computes the same prediction for tgcb's graphs, so that every kernel
the backend runs can be printed beside the time tgc's model gives it, on a ``Machine`` built
from the peaks measured on the B200 the code runs on (``b200``).

What is kept from tgc so the predictions agree with its own: the per-operation costs
(tgc/ir/op.py:201-225: an op missing from the table costs one flop per element, leaves none,
a matmul two per output element and contracted element), and the bytes of a fused execution
(tgc/passes/fusion.py:177-197: chains of single-use elementwise values run as one loop that
reads the chain's outside inputs once and writes its last value once, every other node reads
its inputs and writes its output). ``plan_estimate`` adds the prediction for what the backend
actually moves: the bytes its kernel steps read and write.
"""

from __future__ import annotations

from dataclasses import dataclass

from tgcb.errors import ConfigError

# flops per output element (tgc/ir/op.py:201-225); anything else costs 1.0, leaves 0
OP_FLOPS = {
    "add": 1.0, "sub": 1.0, "mul": 1.0, "div": 4.0, "neg": 1.0, "abs": 1.0, "maximum": 1.0,
    "minimum": 1.0, "relu": 1.0, "reciprocal": 4.0, "exp": 8.0, "log": 8.0, "sqrt": 6.0,
    "tanh": 12.0, "sigmoid": 10.0, "cast": 0.5, "step": 1.0, "sum": 1.0, "mean": 1.0, "max": 1.0,
    "matmul": 2.0, "concat": 0.0, "slice": 0.0,
}


@dataclass
class Machine:
    """An arithmetic peak and a bandwidth (tgc/analysis/cost.py:27-56)."""

    flops_per_second: float = 20e12
    bytes_per_second: float = 1.5e12
    name: str = "reference"

    def __post_init__(self) -> None:
        if self.flops_per_second <= 0 or self.bytes_per_second <= 0:
            raise ConfigError("a machine needs a positive arithmetic peak and a positive bandwidth")

    @property
    def ridge_point(self) -> float:
        """Flops per byte above which a kernel is bound by arithmetic instead of memory."""
        return self.flops_per_second / self.bytes_per_second

    def as_dict(self) -> dict:
        return {"name": self.name, "flops_per_second": self.flops_per_second,
                "bytes_per_second": self.bytes_per_second, "ridge_point": round(self.ridge_point, 2)}


CPU = Machine(500e9, 50e9, "cpu")
GPU = Machine(20e12, 1.5e12, "gpu")  # tgc's placeholder GPU
BANDWIDTH_STARVED = Machine(100e12, 1e12, "bandwidth starved")
MACHINES = {m.name: m for m in (CPU, GPU, BANDWIDTH_STARVED)}

# dense tensor-core rate of each arithmetic kind relative to bf16 on B200 (tf32 : bf16 : int8)
TENSOR_RATE = {"tf32": 0.5, "bf16": 1.0, "int8": 2.0}


# float32 on the CUDA cores (no tensor core): 148 SMs x 128 lanes x 2 flops per fused
# multiply-add x 1.965 GHz; a nominal figure, not a measurement
B200_FP32_SIMT_FLOPS = 148 * 128 * 2 * 1.965e9


def b200(peaks: dict, kind: str = "tf32", sustained: bool = False) -> Machine:
    """The B200 as a roofline machine: the measured copy bandwidth and, for ``kind`` tf32, bf16
    or int8, the dense tensor rate derived from the measured bf16 GEMM rate (burst, or
    ``sustained`` under the power cap); for ``kind`` fp32 the nominal CUDA-core rate (the
    elementwise and reduction kernels). ``peaks`` holds ``hbm_gbs``, ``bf16_tflops`` and
    ``bf16_tflops_sustained``."""
    if kind == "fp32":
        return Machine(B200_FP32_SIMT_FLOPS, peaks["hbm_gbs"] * 1e9, "b200-fp32")
    if kind not in TENSOR_RATE:
        raise ConfigError(f"no B200 rate for {kind!r}; expected fp32 or one of {sorted(TENSOR_RATE)}")
    bf16 = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"]
    return Machine(bf16 * 1e12 * TENSOR_RATE[kind], peaks["hbm_gbs"] * 1e9, f"b200-{kind}")


def get_machine(name: str) -> Machine:
    if name not in MACHINES:
        raise ConfigError(f"unknown machine {name!r}, expected one of {sorted(MACHINES)}")
    return MACHINES[name]


# ----------------------------------------------------------------------------- graph work


def _elements(value) -> int:
    if not value.shape.is_static:
        raise ConfigError(f"{value.name} has a symbolic shape and cannot be costed")
    return value.shape.elements


def node_flops(graph, node) -> float:
    """Arithmetic of one node: per-element cost times output elements; a matmul also times its
    contracted length (the last dimension of its left operand)."""
    if node.op.is_leaf:
        return 0.0
    per = OP_FLOPS.get(node.op.name, 1.0)
    work = per * _elements(node.output)
    if node.op.name == "matmul":
        inner = graph.value(node.inputs[0]).shape.sizes[-1]
        if not inner.is_static:
            raise ConfigError(f"{node.name} contracts a symbolic dimension and cannot be costed")
        work *= inner.value
    return work


def graph_flops(graph) -> float:
    return sum(node_flops(graph, n) for n in graph.nodes)


def chain_groups(graph) -> list[list[str]]:
    """Maximal chains of elementwise nodes that can run as one loop, in tgc's grouping order
    (tgc/passes/fusion.py:70-121): a chain starts at the first ungrouped elementwise node and
    grows while exactly one ungrouped elementwise node reads its last value, that value has no
    other reader and is not a graph output."""
    uses = graph.use_counts()
    outs = set(graph.outputs)
    taken: set[str] = set()
    chains = []
    for node in graph.nodes:
        if node.name in taken or not node.op.is_elementwise:
            continue
        chain = [node.name]
        taken.add(node.name)
        last = node.name
        while uses.get(last, 0) == 1 and last not in outs:
            nxt = [c for c in graph.nodes if c.name not in taken and c.op.is_elementwise and last in c.inputs]
            if len(nxt) != 1:
                break
            chain.append(nxt[0].name)
            taken.add(nxt[0].name)
            last = nxt[0].name
        chains.append(chain)
    return chains


def fused_bytes(graph) -> int:
    """Bytes of tgc's fused execution: each chain reads its outside inputs once and writes its
    last value; every node outside a chain reads its inputs and writes its output."""
    by_name = {n.name: n for n in graph.nodes}
    total = 0
    in_chain: set[str] = set()
    for chain in chain_groups(graph):
        members = set(chain)
        in_chain |= members
        outside: list[str] = []
        for name in chain:
            for operand in by_name[name].inputs:
                if operand not in members and operand not in outside:
                    outside.append(operand)
        total += sum(graph.value(v).bytes for v in outside) + graph.value(chain[-1]).bytes
    for node in graph.nodes:
        if node.name not in in_chain:
            total += sum(graph.value(v).bytes for v in node.inputs) + node.output.bytes
    return total


def unfused_bytes(graph) -> int:
    """Bytes when every node reads its inputs from memory and writes its output there."""
    return sum(sum(graph.value(v).bytes for v in n.inputs) + n.output.bytes for n in graph.nodes)


@dataclass
class RooflineEstimate:
    """Which resource a graph (or plan) runs out of first, and when (tgc/analysis/cost.py:125-177)."""

    flops: float
    bytes_moved: float
    machine: Machine

    @property
    def compute_seconds(self) -> float:
        return self.flops / self.machine.flops_per_second

    @property
    def memory_seconds(self) -> float:
        return self.bytes_moved / self.machine.bytes_per_second

    @property
    def seconds(self) -> float:
        return max(self.compute_seconds, self.memory_seconds)

    @property
    def intensity(self) -> float:
        return self.flops / self.bytes_moved if self.bytes_moved else 0.0

    @property
    def is_memory_bound(self) -> bool:
        return self.intensity < self.machine.ridge_point

    def as_dict(self) -> dict:
        return {"machine": self.machine.name, "flops": self.flops, "bytes": self.bytes_moved,
                "intensity": round(self.intensity, 4), "seconds": self.seconds, "memory_bound": self.is_memory_bound}


def estimate(graph, machine: Machine = GPU, *, fused: bool = True) -> RooflineEstimate:
    """tgc's prediction for a graph: its flops, and the bytes of tgc's fused (or unfused) execution."""
    moved = fused_bytes(graph) if fused else unfused_bytes(graph)
    return RooflineEstimate(graph_flops(graph), float(moved), machine)


def plan_estimate(compiled, machine: Machine) -> RooflineEstimate:
    """The same roofline for what the backend runs: the graph's flops against the bytes its
    kernel steps read and write (each materialised value once per step that touches it)."""
    low = compiled.lowering
    moved = 0
    for step in compiled.module.steps:
        moved += sum(low.values[r].bytes for r in step.reads if r in low.values)
        moved += sum(low.values[w].bytes for w in step.writes if w in low.values)
    return RooflineEstimate(graph_flops(compiled.graph), float(moved), machine)
