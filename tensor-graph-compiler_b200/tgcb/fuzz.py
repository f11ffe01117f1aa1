"""Generated graphs, compiled by tgcb and run on the GPU, against a reference executor.

Restates tgc/verify/fuzz.py for this backend. ``generate`` is tgc's generator step for step
(fuzz.py:67-104: one ``random.Random(seed)``, values kept at the full [rows, columns] shape
or a [rows, 1] column, the same choices drawn in the same order), so seed s gives the graph
tgc's fuzzer gives, name for name. ``fuzz_compiler`` (fuzz.py:361-385) compiles each graph
with ``tgcb.runtime.compile_graph`` and compares the GPU's outputs with ``reference(graph,
feeds)``; tgc compares against its own interpreter, and callers pass one in (the library does
not ship an interpreter). The GPU's tanh/sigmoid/exp and its row-reduction order differ from
ATen's in the last bits, so the comparison is ``outputs_agree`` at a tolerance instead of bit
equality. ``shrink`` (fuzz.py:210-270) removes nodes while a failure survives.
``fuzz_allocation`` (fuzz.py:388-407) checks every generated graph's arena plan over the
kernel steps this backend runs.
"""

from __future__ import annotations

import random
from collections.abc import Callable
from dataclasses import dataclass, field

import torch

from tgcb import ir, memory
from tgcb.errors import ConfigError, VerificationError

ELEMENTWISE_UNARY = ("relu", "tanh", "neg", "sigmoid", "abs")
ELEMENTWISE_BINARY = ("add", "sub", "mul", "maximum", "minimum")
DEFAULT_TOLERANCE = 1e-5


@dataclass(frozen=True)
class GeneratorConfig:
    """The generator's knobs, under the names tgc's fuzzer takes them (fuzz.py:37-64): graph
    size (nodes drawn, inputs declared), the [rows, columns] every full value has, and the
    odds of drawing a row reduction and of reusing one operand for both sides of a binary op."""

    nodes: int = 12
    inputs: int = 2
    rows: int = 8
    columns: int = 8
    reduction_chance: float = 0.15
    reuse_chance: float = 0.3

    def __post_init__(self) -> None:
        bad = [f"{k}={getattr(self, k)} (at least 1)" for k in ("nodes", "inputs") if getattr(self, k) < 1]
        bad += [f"{k}={getattr(self, k)} (a probability, 0 to 1)" for k in ("reduction_chance", "reuse_chance")
                if not 0.0 <= getattr(self, k) <= 1.0]
        if bad:
            raise ConfigError("unusable generator settings: " + ", ".join(bad))

    def as_dict(self) -> dict:
        return {"nodes": self.nodes, "inputs": self.inputs, "shape": [self.rows, self.columns],
                "reduction_chance": self.reduction_chance}


def generate(config: GeneratorConfig | None = None, seed: int = 0) -> ir.Graph:
    """A random graph of elementwise operations, row sums and broadcasts (fuzz.py:67-104)."""
    cfg = config or GeneratorConfig()
    rng = random.Random(seed)
    b = ir.Builder()
    full: list[str] = [b.input([cfg.rows, cfg.columns], name=f"in{i}") for i in range(cfg.inputs)]
    columns: list[str] = []
    for _ in range(cfg.nodes):
        if columns and rng.random() < 0.2:
            full.append(b.broadcast_to(rng.choice(columns), [cfg.rows, cfg.columns]))
            continue
        if rng.random() < cfg.reduction_chance:
            columns.append(b.sum(rng.choice(full), axes=[1], keepdims=True))
            continue
        if rng.random() < 0.4:
            src = rng.choice(full)
            full.append(b.apply(ir.get_op(rng.choice(ELEMENTWISE_UNARY)), src))
            continue
        left = rng.choice(full)
        right = rng.choice(full) if rng.random() > cfg.reuse_chance else left
        full.append(b.apply(ir.get_op(rng.choice(ELEMENTWISE_BINARY)), left, right))
    return b.finish(full[-1])


def generate_many(count: int = 50, config: GeneratorConfig | None = None, start: int = 0) -> list[ir.Graph]:
    if count < 1:
        raise ConfigError(f"the count must be positive, got {count}")
    return [generate(config, seed=start + i) for i in range(count)]


def feeds_for(graph: ir.Graph, seed: int = 0) -> dict[str, torch.Tensor]:
    """tgc's random_feeds(graph, seed=seed, positive=True) for float32 inputs
    (reference.py:174-205): one seeded generator, randn per input in declaration order, |x|+0.5."""
    g = torch.Generator().manual_seed(seed)
    feeds = {}
    for v in graph.inputs:
        if v.dtype.name != "float32":
            raise ConfigError(f"generated graphs take float32 inputs, {v.name} is {v.dtype.name}")
        sizes = list(v.shape.ints())
        feeds[v.name] = torch.randn(sizes, generator=g, dtype=torch.float32).abs() + 0.5
    return feeds


def outputs_agree(left, right, *, tolerance: float = 0.0) -> bool:
    """Bit equality at tolerance 0, else allclose with atol = rtol = tolerance (reference.py:208-227)."""
    if len(left) != len(right):
        return False
    for a, b in zip(left, right, strict=True):
        a, b = a.detach().cpu(), b.detach().cpu()
        if a.shape != b.shape:
            return False
        if tolerance == 0.0:
            if not torch.equal(a, b):
                return False
        elif not torch.allclose(a.float(), b.float(), atol=tolerance, rtol=tolerance):
            return False
    return True


@dataclass(frozen=True)
class Failure:
    """A generated graph the backend got wrong: the seed that drew it, the graph (shrunk, when
    shrinking ran) and what went wrong."""

    seed: int
    graph: ir.Graph
    detail: str = ""

    def as_dict(self) -> dict:
        return {"seed": self.seed, "nodes": len(self.graph.nodes), "detail": self.detail}


@dataclass
class FuzzReport:
    checked: int = 0
    failures: list[Failure] = field(default_factory=list)

    @property
    def passed(self) -> int:
        return self.checked - len(self.failures)

    @property
    def clean(self) -> bool:
        return not self.failures

    def as_dict(self) -> dict:
        return {
            "checked": self.checked,
            "passed": self.passed,
            "failures": len(self.failures),
            "smallest_failure": min((len(f.graph.nodes) for f in self.failures), default=0),
        }


Reference = Callable[[ir.Graph, dict], list]


def compiled_outputs(graph: ir.Graph, feeds: dict, device: int | None = None) -> list[torch.Tensor]:
    """Compile with tgcb and run once on the GPU; outputs copied to the host."""
    from tgcb.runtime import compile_graph

    dev = torch.cuda.current_device() if device is None else device
    compiled = compile_graph(graph, device=dev)
    outs = compiled({k: v.cuda(dev) for k, v in feeds.items()})
    torch.cuda.synchronize(dev)
    compiled.check_status()
    return [o.detach().cpu().clone() for o in outs]


def check_one(graph: ir.Graph, seed: int, reference: Reference, tolerance: float, device: int | None = None) -> str:
    """'' when the GPU agrees with the reference on feeds_for(graph, seed), else why not."""
    feeds = feeds_for(graph, seed)
    try:
        produced = compiled_outputs(graph, feeds, device)
        expected = reference(graph, feeds)
    except Exception as failure:  # noqa: BLE001 - a compile or run error is a finding
        return f"raised {type(failure).__name__}: {failure}"
    if len(produced) != len(expected) or any(a.shape != b.shape for a, b in zip(produced, expected, strict=True)):
        return "produced outputs of other shapes than the reference"
    if not outputs_agree(produced, expected, tolerance=tolerance):
        worst = max(
            float((a.double() - b.detach().cpu().double()).abs().max()) if a.numel() else 0.0
            for a, b in zip(produced, expected, strict=True)
        )
        return f"disagreed (largest difference {worst:.3g})"
    return ""


def fuzz_compiler(
    count: int = 30,
    config: GeneratorConfig | None = None,
    *,
    reference: Reference,
    tolerance: float = DEFAULT_TOLERANCE,
    start: int = 0,
    device: int | None = None,
) -> FuzzReport:
    """Compile and run generated graphs on the GPU, each checked against ``reference``."""
    if count < 1:
        raise ConfigError(f"the count must be positive, got {count}")
    report = FuzzReport()
    for seed in range(start, start + count):
        graph = generate(config, seed=seed)
        report.checked += 1
        detail = check_one(graph, seed, reference, tolerance, device)
        if detail:
            report.failures.append(Failure(seed=seed, graph=graph, detail=detail))
    return report


def drop_node(graph: ir.Graph, index: int) -> ir.Graph | None:
    """The graph without one node, its readers rewired to its first input (fuzz.py:245-270);
    None when that breaks the graph or changes an output's shape."""
    node = graph.nodes[index]
    if not node.inputs:
        return None
    replacement = {node.name: node.inputs[0]}
    kept = [other.replace_inputs(replacement) for pos, other in enumerate(graph.nodes) if pos != index]
    outputs = [replacement.get(n, n) for n in graph.outputs]
    candidate = ir.Graph(nodes=kept, inputs=list(graph.inputs), outputs=outputs)
    try:
        ir.validate(candidate)
    except Exception:  # noqa: BLE001 - any invalid candidate is skipped
        return None
    if any(graph.value(n).shape != candidate.value(n).shape for n in candidate.outputs):
        return None
    return candidate


def shrink(graph: ir.Graph, fails: Callable[[ir.Graph], bool], *, rounds: int = 32) -> ir.Graph:
    """Remove nodes while ``fails`` still holds, greedily, until none can go (fuzz.py:210-242)."""
    if rounds < 1:
        raise ConfigError(f"the round count must be positive, got {rounds}")
    if not fails(graph):
        raise VerificationError("this graph does not fail, so there is nothing to shrink")
    current = graph
    for _ in range(rounds):
        smaller = None
        for index in range(len(current.nodes)):
            candidate = drop_node(current, index)
            if candidate is not None and fails(candidate):
                smaller = candidate
                break
        if smaller is None:
            return current
        current = smaller
    return current


def fuzz_allocation(count: int = 40, config: GeneratorConfig | None = None) -> FuzzReport:
    """Every generated graph's arena plan, over the kernel steps tgcb lowers it to, keeps
    live values apart (the check of fuzz.py:388-407 on this backend's planner)."""
    from tgcb import runtime

    if count < 1:
        raise ConfigError(f"the count must be positive, got {count}")
    report = FuzzReport()
    for seed in range(count):
        graph = generate(config, seed=seed)
        report.checked += 1
        try:
            og, _order, plan, mod, low = runtime.generate(graph)
            sizes = {v.name: v.bytes for v in og.inputs}
            for s in mod.steps:
                for w in s.writes:
                    sizes[w] = low.scratch.get(w, low.values[w].bytes if w in low.values else 0)
            iv = memory.intervals_for_steps(low.inputs, [(s.reads, s.writes) for s in mod.steps], low.outputs, sizes)
            memory.validate_plan(iv, plan)
        except Exception as failure:  # noqa: BLE001 - any planning error is a finding
            report.failures.append(Failure(seed=seed, graph=graph, detail=str(failure)))
    return report


def generated_graph_statistics(count: int = 50, config: GeneratorConfig | None = None) -> dict:
    """What the generator produces (fuzz.py:316-334)."""
    if count < 1:
        raise ConfigError(f"the count must be positive, got {count}")
    reductions = reused = 0
    sizes = []
    for seed in range(count):
        graph = generate(config, seed=seed)
        sizes.append(len(graph.nodes))
        reductions += sum(1 for n in graph.nodes if n.op.name == "sum")
        reused += sum(1 for _, uses in graph.use_counts().items() if uses > 1)
    return {"graphs": count, "mean_nodes": round(sum(sizes) / count, 2), "reductions": reductions,
            "values_read_more_than_once": reused}
