"""Reverse mode: the graph that computes gradients of a scalar graph output.

A restatement of tgc/grad/reverse.py:70-224 and the per-op rules of tgc/grad/rules.py:96-396,
so the training-step workload (the gradient of an MLP's mean-squared error) can be built
where tgc is not installed. The rules issue the same builder calls in the same order as
tgc's, so a gradient graph printed by tgcb and by tgc is the same text, value names included;
tests/test_grad.py checks that against graphs tgc produced. The result is an ordinary graph
that ``tgcb.runtime.compile_graph`` lowers like any other: matmuls (with their transposes
folded into operand majors) become tcgen05 GEMMs, broadcast gradients become column sums.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass

from tgcb import ir
from tgcb.errors import ConfigError, PassError

COTANGENT = "cotangent"
NON_DIFFERENTIABLE = {"input", "constant", "step", "cast"}


@dataclass
class GradientResult:
    graph: ir.Graph
    forward_nodes: int
    backward_nodes: int
    wrt: tuple[str, ...] = ()


class _Ctx:
    def __init__(self, node, cotangent: str, operands: list[str], output: str, shapes: list):
        self.node = node
        self.cotangent = cotangent
        self.operands = operands
        self.output = output
        self.shapes = shapes

    @property
    def attrs(self) -> dict:
        return self.node.attrs


def _sizes(shape) -> list[int]:
    out = []
    for d in shape.sizes:
        if not d.is_static:
            raise PassError(f"cannot differentiate through the symbolic dimension {d.name}")
        out.append(d.value)
    return out


def sum_to_shape(b: ir.Builder, name: str, source, target) -> str:
    """Undo broadcasting on a cotangent: sum it over every axis that broadcasting created
    (leading axes the operand lacks) or widened (the operand's size-1 axes), in increasing axis
    order with the dimensions kept, then drop the leading ones with a reshape. These are the
    builder calls tgc/grad/rules.py:96-128 makes, so gradient graphs print alike."""
    have, want = _sizes(source), _sizes(target)
    if have == want:
        return name
    lead = len(have) - len(want)
    if lead < 0:
        raise PassError(f"cannot reduce a rank-{len(have)} cotangent to rank {len(want)}")
    padded = [1] * lead + list(want)
    axes = []
    for axis, (h, w) in enumerate(zip(have, padded, strict=True)):
        if axis < lead or (w == 1 and h != 1):
            axes.append(axis)
        elif w != h:
            raise PassError(f"shape {have} was not broadcast from {want}")
    out = b.sum(name, axes=axes, keepdims=True) if axes else name
    return out if _sizes(b.shape_of(out)) == want else b.reshape(out, want)


def _binary_sum(b, ctx, left, right):
    return [
        sum_to_shape(b, left, b.shape_of(left), ctx.shapes[0]),
        sum_to_shape(b, right, b.shape_of(right), ctx.shapes[1]),
    ]


def _add(b, c):
    g = c.cotangent
    out = b.shape_of(g)
    return [sum_to_shape(b, g, out, c.shapes[0]), sum_to_shape(b, g, out, c.shapes[1])]


def _sub(b, c):
    g = c.cotangent
    out = b.shape_of(g)
    neg = b.neg(g)
    return [sum_to_shape(b, g, out, c.shapes[0]), sum_to_shape(b, neg, out, c.shapes[1])]


def _mul(b, c):
    left = b.mul(c.cotangent, c.operands[1])
    right = b.mul(c.cotangent, c.operands[0])
    return _binary_sum(b, c, left, right)


def _div(b, c):
    left = b.div(c.cotangent, c.operands[1])
    scaled = b.mul(c.cotangent, c.output)
    right = b.neg(b.div(scaled, c.operands[1]))
    return _binary_sum(b, c, left, right)


def _neg(b, c):
    return [b.neg(c.cotangent)]


def _exp(b, c):
    return [b.mul(c.cotangent, c.output)]


def _log(b, c):
    return [b.div(c.cotangent, c.operands[0])]


def _sqrt(b, c):
    half = b.constant(0.5, dtype=c.node.output.dtype)
    return [b.mul(b.div(c.cotangent, c.output), half)]


def _reciprocal(b, c):
    sq = b.mul(c.output, c.output)
    return [b.neg(b.mul(c.cotangent, sq))]


def _tanh(b, c):
    one = b.constant(1.0, dtype=c.node.output.dtype)
    sq = b.mul(c.output, c.output)
    return [b.mul(c.cotangent, b.sub(one, sq))]


def _sigmoid(b, c):
    one = b.constant(1.0, dtype=c.node.output.dtype)
    comp = b.sub(one, c.output)
    return [b.mul(c.cotangent, b.mul(c.output, comp))]


def _relu(b, c):
    return [b.mul(c.cotangent, b.step(c.operands[0]))]


def _abs(b, c):
    pos = b.step(c.operands[0])
    neg = b.step(b.neg(c.operands[0]))
    return [b.mul(c.cotangent, b.sub(pos, neg))]


def _pick(b, c, first: int, second: int):
    one = b.constant(1.0, dtype=c.node.output.dtype)
    picked = b.step(b.sub(c.operands[first], c.operands[second]))
    left = b.mul(c.cotangent, picked)
    right = b.mul(c.cotangent, b.sub(one, picked))
    return _binary_sum(b, c, left, right)


def _maximum(b, c):
    return _pick(b, c, 0, 1)


def _minimum(b, c):
    return _pick(b, c, 1, 0)


def _reduced(c) -> tuple[list[int], list[int]]:
    axes = sorted(int(a) for a in c.attrs["axes"])
    sizes = _sizes(c.shapes[0])
    keep = bool(c.attrs.get("keepdims", False))
    mid = list(sizes)
    for a in axes:
        mid[a] = 1
    return (mid if not keep else [], sizes)


def _sum(b, c):
    mid, sizes = _reduced(c)
    g = c.cotangent
    if mid:
        g = b.reshape(g, mid)
    return [b.broadcast_to(g, sizes)]


def _mean(b, c):
    mid, sizes = _reduced(c)
    divisor = 1
    for a in sorted(int(a) for a in c.attrs["axes"]):
        divisor *= sizes[a]
    g = c.cotangent
    if mid:
        g = b.reshape(g, mid)
    scale = b.constant(1.0 / divisor, dtype=c.node.output.dtype)
    return [b.broadcast_to(b.mul(g, scale), sizes)]


def _max(b, c):
    mid, sizes = _reduced(c)
    g, peak = c.cotangent, c.output
    if mid:
        g = b.reshape(g, mid)
        peak = b.reshape(peak, mid)
    one = b.constant(1.0, dtype=c.node.output.dtype)
    wide = b.broadcast_to(peak, sizes)
    gap = b.sub(wide, c.operands[0])
    mask = b.sub(one, b.step(gap))
    return [b.mul(b.broadcast_to(g, sizes), mask)]


def _matmul(b, c):
    if len(_sizes(c.shapes[0])) != 2 or len(_sizes(c.shapes[1])) != 2:
        raise PassError("the matmul rule handles rank two")
    right_t = b.transpose(c.operands[1], [1, 0])
    left_t = b.transpose(c.operands[0], [1, 0])
    return [b.matmul(c.cotangent, right_t), b.matmul(left_t, c.cotangent)]


def _transpose(b, c):
    perm = [int(a) for a in c.attrs["permutation"]]
    inv = [0] * len(perm)
    for pos, a in enumerate(perm):
        inv[a] = pos
    return [b.transpose(c.cotangent, inv)]


def _reshape(b, c):
    return [b.reshape(c.cotangent, _sizes(c.shapes[0]))]


def _broadcast(b, c):
    g = c.cotangent
    return [sum_to_shape(b, g, b.shape_of(g), c.shapes[0])]


def _concat(b, c):
    axis = int(c.attrs["axis"])
    left = _sizes(c.shapes[0])[axis]
    right = _sizes(c.shapes[1])[axis]
    return [b.slice(c.cotangent, axis, 0, left), b.slice(c.cotangent, axis, left, right)]


def _slice(b, c):
    axis, start, length = int(c.attrs["axis"]), int(c.attrs["start"]), int(c.attrs["length"])
    sizes = _sizes(c.shapes[0])
    dt = c.node.output.dtype
    cur = c.cotangent
    if start:
        before = list(sizes)
        before[axis] = start
        cur = b.concat(b.broadcast_to(b.constant(0.0, dtype=dt), before), cur, axis)
    trailing = sizes[axis] - start - length
    if trailing:
        after = list(sizes)
        after[axis] = trailing
        cur = b.concat(cur, b.broadcast_to(b.constant(0.0, dtype=dt), after), axis)
    return [cur]


def _identity(b, c):
    return [c.cotangent]


RULES: dict[str, Callable] = {
    "add": _add, "sub": _sub, "mul": _mul, "div": _div, "neg": _neg, "exp": _exp, "log": _log,
    "sqrt": _sqrt, "reciprocal": _reciprocal, "tanh": _tanh, "sigmoid": _sigmoid, "relu": _relu,
    "abs": _abs, "maximum": _maximum, "minimum": _minimum, "sum": _sum, "mean": _mean, "max": _max,
    "matmul": _matmul, "transpose": _transpose, "reshape": _reshape, "broadcast_to": _broadcast,
    "concat": _concat, "slice": _slice, "print": _identity, "assert_finite": _identity,
}


def _needed(graph, output: str, wrt: Sequence[str]) -> set[str]:
    reaching = set(wrt)
    for n in graph.nodes:
        if any(i in reaching for i in n.inputs):
            reaching.add(n.name)
    reached = {output}
    for n in reversed(graph.nodes):
        if n.name in reached:
            reached.update(n.inputs)
    return reaching & reached


def gradient(graph, wrt: Sequence[str] | None = None, *, keep_forward: bool = False, seed_is_input: bool = True) -> GradientResult:
    """Gradients of the single output of ``graph`` w.r.t. ``wrt`` (tgc/grad/reverse.py:149-224)."""
    if len(graph.outputs) != 1:
        raise ConfigError(f"a gradient needs exactly one output, got {len(graph.outputs)}")
    blocking = sorted({n.op.name for n in graph.nodes if n.op.name not in RULES and n.op.name not in ("input", "constant")})
    if blocking:
        raise ConfigError(f"these operations have no gradient rule: {blocking}")
    targets = list(wrt) if wrt is not None else [v.name for v in graph.inputs]
    if not targets:
        raise ConfigError("there is nothing to differentiate with respect to")
    known = {v.name for v in graph.inputs}
    unknown = [t for t in targets if t not in known]
    if unknown:
        raise ConfigError(f"{unknown} are not inputs of this graph")
    if seed_is_input and COTANGENT in known:
        raise ConfigError(f"the graph already has an input named {COTANGENT!r}")

    b = ir.Builder()
    mapping: dict[str, str] = {}
    for v in graph.inputs:
        mapping[v.name] = b.input([d.value if d.is_static else d.name for d in v.shape.sizes], dtype=v.dtype, name=v.name)
    for n in graph.nodes:
        if n.op.name == "constant":
            mapping[n.name] = b.constant(float(n.attrs["value"]), dtype=n.output.dtype)
            continue
        mapping[n.name] = b.apply(ir.get_op(n.op.name), *[mapping[i] for i in n.inputs], **n.attrs)
    forward_nodes = len(b.nodes)

    output = graph.outputs[0]
    needed = _needed(graph, output, targets)
    out_name = mapping[output]
    sizes = _sizes(b.shape_of(out_name))
    if seed_is_input:
        seed = b.input(sizes, dtype=b.dtype_of(out_name), name=COTANGENT)
    else:
        one = b.constant(1.0, dtype=b.dtype_of(out_name))
        seed = b.broadcast_to(one, sizes) if sizes else one
    cot: dict[str, str] = {output: seed}
    values = {v.name: v for v in graph.inputs} | {n.name: n.output for n in graph.nodes}
    for n in reversed(graph.nodes):
        if n.name not in cot or n.name not in needed or n.op.name not in RULES:
            continue
        ctx = _Ctx(n, cot[n.name], [mapping[i] for i in n.inputs], mapping[n.name], [values[i].shape for i in n.inputs])
        for name, contribution in zip(n.inputs, RULES[n.op.name](b, ctx), strict=True):
            if contribution is None or name not in needed:
                continue
            cot[name] = b.add(cot[name], contribution) if name in cot else contribution
    missing = [t for t in targets if t not in cot]
    if missing:
        raise PassError(f"{missing} do not reach the output, so they have no gradient")
    outs = [mapping[output]] if keep_forward else []
    outs.extend(cot[t] for t in targets)
    result = b.finish(*outs)
    return GradientResult(result, forward_nodes, len(result.nodes) - forward_nodes, tuple(targets))
