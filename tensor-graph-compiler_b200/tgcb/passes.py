"""The exact pass pipeline that runs before lowering.

tgc's executor runs five passes to a fixed point before it generates code
(tgc/runtime/executor.py:33-48): scalar constant folding, the exact algebraic identities,
transpose cancellation, common subexpressions and dead code. Each preserves the answer bit
for bit, which is why the compiled graph can be held to the interpreter. They are restated
here so a graph compiles identically where tgc is absent; when tgc is present its own
``Pipeline`` may be passed to ``tgcb.runtime.compile_graph`` instead.

Reference map:
  fold_constants ......... tgc/passes/constfold.py:50-183 (scalar-only, in the declared type)
  simplify ............... tgc/passes/algebraic.py:62-239 (EXACT_RULES only)
  cancel_transposes ...... tgc/passes/layout.py:127-165
  CSE .................... tgc/passes/cse.py:43-77
  DCE .................... tgc/passes/dce.py:40-66
  Pass / Pipeline ........ tgc/passes/manager.py:88-213
"""

from __future__ import annotations

import math
import struct
from collections.abc import Callable
from dataclasses import dataclass, field

from tgcb import ir
from tgcb.errors import ConfigError, PassError

Transform = Callable[[ir.Graph], ir.Graph]

# ----------------------------------------------------------------------------- constant folding

_UNARY_FOLDS = {
    "neg": lambda x: -x,
    "abs": abs,
    "exp": math.exp,
    "log": math.log,
    "sqrt": math.sqrt,
    "tanh": math.tanh,
    "relu": lambda x: max(0.0, x),
    "sigmoid": lambda x: 1.0 / (1.0 + math.exp(-x)),
    "reciprocal": lambda x: 1.0 / x,
    "step": lambda x: 1.0 if x > 0 else 0.0,
}
_BINARY_FOLDS = {
    "add": lambda a, b: a + b,
    "sub": lambda a, b: a - b,
    "mul": lambda a, b: a * b,
    "div": lambda a, b: a / b,
    "maximum": max,
    "minimum": min,
}


def round_to(value: float, dtype: ir.DType) -> float:
    """``value`` as ``dtype`` stores it: through struct for 16/32-bit floats, int() for ints."""
    if not dtype.is_float:
        return float(int(value))
    if dtype is ir.FLOAT64:
        return value
    code = "e" if dtype.bits == 16 else "f"
    try:
        return struct.unpack(code, struct.pack(code, value))[0]
    except OverflowError:
        return math.copysign(math.inf, value)


def _foldable_into(value: float, dtype: ir.DType) -> bool:
    if math.isnan(value) or math.isinf(value):
        return False
    if dtype.is_integral:
        return value == int(value) and ir.can_represent_exactly(dtype, int(value))
    return not math.isinf(round_to(value, dtype))


def fold_constants(graph: ir.Graph) -> ir.Graph:
    """Replace rank-0 nodes whose operands are all literals by the literal they produce."""
    known = {n.name: float(n.attrs["value"]) for n in graph.nodes if n.op is ir.CONSTANT}
    kept: list[ir.Node] = []
    for n in graph.nodes:
        name = n.op.name
        foldable = (
            n.op is not ir.CONSTANT
            and n.op.pure
            and (name in _UNARY_FOLDS or name in _BINARY_FOLDS or name == "cast")
            and n.output.shape.rank == 0
            and all(i in known for i in n.inputs)
        )
        if not foldable:
            kept.append(n)
            continue
        args = [known[i] for i in n.inputs]
        try:
            if name in _UNARY_FOLDS:
                value = float(_UNARY_FOLDS[name](args[0]))
            elif name in _BINARY_FOLDS:
                value = float(_BINARY_FOLDS[name](args[0], args[1]))
            else:
                value = round_to(args[0], n.output.dtype)
        except (ValueError, ZeroDivisionError, OverflowError):
            kept.append(n)
            continue
        if not _foldable_into(value, n.output.dtype):
            kept.append(n)
            continue
        folded = round_to(value, n.output.dtype)
        known[n.name] = folded
        kept.append(ir.Node(ir.CONSTANT, (), n.output, {"value": folded}))
    return graph.with_nodes(kept)


# ----------------------------------------------------------------------------- exact algebra


def _exact_identity(node: ir.Node, constants: dict[str, float], producers: dict[str, ir.Node]) -> str | None:
    """The operand ``node`` reduces to under an exact rule, if any.

    The five rules tgc marks exact, tried in its order: x*1, x/1, x+0, x-0, -(-x).
    """
    op = node.op
    if op is ir.MUL:
        a, b = node.inputs
        if constants.get(b) == 1.0:
            return a
        if constants.get(a) == 1.0:
            return b
        return None
    if op is ir.DIV:
        a, b = node.inputs
        return a if constants.get(b) == 1.0 else None
    if op is ir.ADD:
        a, b = node.inputs
        if constants.get(b) == 0.0:
            return a
        if constants.get(a) == 0.0:
            return b
        return None
    if op is ir.SUB:
        a, b = node.inputs
        return a if constants.get(b) == 0.0 else None
    if op is ir.NEG:
        inner = producers.get(node.inputs[0])
        if inner is not None and inner.op is ir.NEG:
            return inner.inputs[0]
    return None


def simplify(graph: ir.Graph) -> ir.Graph:
    """Drop nodes that are an exact identity of one of their operands."""
    constants = {n.name: float(n.attrs["value"]) for n in graph.nodes if n.op is ir.CONSTANT}
    producers = {n.name: n for n in graph.nodes}
    replacement: dict[str, str] = {}
    kept: list[ir.Node] = []
    for n in graph.nodes:
        r = n.replace_inputs(replacement)
        producers[n.name] = r
        target = _exact_identity(r, constants, producers)
        if target is None:
            kept.append(r)
        else:
            replacement[n.name] = replacement.get(target, target)
    outputs = [replacement.get(o, o) for o in graph.outputs]
    return ir.Graph(kept, list(graph.inputs), outputs)


# ----------------------------------------------------------------------------- transposes


def _compose(outer, inner) -> tuple[int, ...]:
    if len(outer) != len(inner):
        raise ConfigError("two permutations of different ranks do not compose")
    return tuple(inner[a] for a in outer)


def cancel_transposes(graph: ir.Graph) -> ir.Graph:
    """Merge transpose-of-transpose into one, or drop it when the composition is identity."""
    producers = {n.name: n for n in graph.nodes}
    replacement: dict[str, str] = {}
    kept: list[ir.Node] = []
    for n in graph.nodes:
        r = n.replace_inputs(replacement)
        producers[n.name] = r
        if r.op is not ir.TRANSPOSE:
            kept.append(r)
            continue
        inner = producers.get(r.inputs[0])
        if inner is None or inner.op is not ir.TRANSPOSE:
            kept.append(r)
            continue
        combined = _compose(r.attrs["permutation"], inner.attrs["permutation"])
        if combined == tuple(range(len(combined))):
            replacement[n.name] = replacement.get(inner.inputs[0], inner.inputs[0])
            continue
        merged = ir.Node(ir.TRANSPOSE, inner.inputs, r.output, {"permutation": combined})
        producers[n.name] = merged
        kept.append(merged)
    outputs = [replacement.get(o, o) for o in graph.outputs]
    return ir.Graph(kept, list(graph.inputs), outputs)


# ----------------------------------------------------------------------------- CSE / DCE


def eliminate_common_subexpressions(graph: ir.Graph) -> ir.Graph:
    """Keep the first of every set of pure non-leaf nodes with equal signatures."""
    seen: dict[tuple, str] = {}
    replacement: dict[str, str] = {}
    kept: list[ir.Node] = []
    for n in graph.nodes:
        r = n.replace_inputs(replacement)
        if not (n.op.pure and not n.op.is_leaf):
            kept.append(r)
            continue
        key = r.signature()
        if key in seen:
            replacement[n.name] = seen[key]
            continue
        seen[key] = n.name
        kept.append(r)
    outputs = [replacement.get(o, o) for o in graph.outputs]
    return ir.Graph(kept, list(graph.inputs), outputs)


def live_values(graph: ir.Graph) -> set[str]:
    """Outputs and side effects, closed backwards over inputs."""
    live = set(ir.reachable_from_outputs(graph))
    for n in graph.nodes:
        if not n.op.can_be_removed_if_unused:
            live.add(n.name)
    changed = True
    while changed:
        changed = False
        for n in reversed(graph.nodes):
            if n.name in live:
                for i in n.inputs:
                    if i not in live:
                        live.add(i)
                        changed = True
    return live


def eliminate_dead_code(graph: ir.Graph) -> ir.Graph:
    live = live_values(graph)
    return graph.with_nodes([n for n in graph.nodes if n.name in live])


# ----------------------------------------------------------------------------- pipeline


def graphs_equal(left: ir.Graph, right: ir.Graph) -> bool:
    """Structural node-for-node equality (tgc/passes/manager.py:122-137)."""
    if len(left.nodes) != len(right.nodes) or list(left.outputs) != list(right.outputs):
        return False
    for a, b in zip(left.nodes, right.nodes, strict=True):
        if a.op.name != b.op.name or tuple(a.inputs) != tuple(b.inputs):
            return False
        if a.output != b.output or a.attrs != b.attrs:
            return False
    return True


@dataclass
class PassResult:
    name: str
    nodes_before: int
    nodes_after: int
    changed: bool


@dataclass
class Pass:
    name: str
    transform: Transform
    enabled: bool = True

    def run(self, graph: ir.Graph, *, check: bool = True) -> tuple[ir.Graph, PassResult]:
        before = len(graph.nodes)
        out = self.transform(graph)
        if check:
            try:
                ir.validate(out)
            except Exception as failure:  # noqa: BLE001 - re-raised with the pass named
                raise PassError(f"{self.name} produced an invalid graph: {failure}") from failure
        return out, PassResult(self.name, before, len(out.nodes), not graphs_equal(graph, out))


@dataclass
class PipelineReport:
    results: list[PassResult] = field(default_factory=list)
    rounds: int = 0


@dataclass
class Pipeline:
    """Passes run in order, repeatedly, until a round changes nothing (tgc/passes/manager.py:140-213)."""

    passes: list[Pass] = field(default_factory=list)
    max_rounds: int = 8
    check_after_each: bool = True

    def run(self, graph: ir.Graph) -> tuple[ir.Graph, PipelineReport]:
        ir.validate(graph)
        report = PipelineReport()
        current = graph
        for r in range(self.max_rounds):
            report.rounds = r + 1
            changed = False
            for p in self.passes:
                if not p.enabled:
                    continue
                current, res = p.run(current, check=self.check_after_each)
                report.results.append(res)
                changed = changed or res.changed
            if not changed:
                return current, report
        raise PassError(
            f"the pipeline was still changing the graph after {self.max_rounds} rounds, "
            f"which means two of {[p.name for p in self.passes if p.enabled]} are undoing each other"
        )


def default_pipeline() -> Pipeline:
    """The five exact passes in tgc's order (tgc/runtime/executor.py:33-48)."""
    return Pipeline(
        [
            Pass("constant folding", fold_constants),
            Pass("algebraic", simplify),
            Pass("transposes", cancel_transposes),
            Pass("subexpressions", eliminate_common_subexpressions),
            Pass("dead code", eliminate_dead_code),
        ]
    )
