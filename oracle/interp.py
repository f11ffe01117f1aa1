"""Restatement of tgc's reference interpreter and of its generated-Python executor. TEST ONLY.

``run`` / ``interpret`` follow tgc/verify/reference.py:74-171 op for op with the same torch
CPU kernels, so on the same torch build they give tgc's own numbers; the golden fixtures
pin that. ``ArenaProgram`` follows tgc/codegen/emit.py:92-209 (each value a typed view of one
zeroed arena at its planned offset, inputs copied in, one ``copy_`` of a torch op per node,
outputs returned as views) and is the CPU baseline the benchmark times.

Graphs are read duck-typed (``nodes``, ``inputs``, ``outputs``, ``op.name``, ``attrs``), so
tgc's ``Graph`` and tgcb's mirror both work.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

TORCH = {
    "bool": torch.bool,
    "int8": torch.int8,
    "int32": torch.int32,
    "int64": torch.int64,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float32": torch.float32,
    "float64": torch.float64,
}

_UNARY = {
    "neg": torch.neg,
    "exp": torch.exp,
    "log": torch.log,
    "sqrt": torch.sqrt,
    "tanh": torch.tanh,
    "relu": torch.relu,
    "sigmoid": torch.sigmoid,
    "reciprocal": torch.reciprocal,
    "abs": torch.abs,
    "step": lambda t: (t > 0).to(t.dtype),
}
_BINARY = {
    "add": torch.add,
    "sub": torch.sub,
    "mul": torch.mul,
    "div": torch.div,
    "maximum": torch.maximum,
    "minimum": torch.minimum,
}


def _sizes(value) -> tuple[int, ...]:
    return tuple(int(d.value or 0) for d in value.shape.sizes)


def _reduce(node, src: torch.Tensor) -> torch.Tensor:
    """reference.py:115-128: widen to the accumulator dtype; max via amax axis by axis."""
    axes = tuple(node.attrs["axes"])
    keep = bool(node.attrs.get("keepdims", False))
    acc = TORCH[node.output.dtype.name]
    if node.op.name == "max":
        out = src
        for a in sorted(axes, reverse=True):
            out = out.amax(dim=a, keepdim=True)
        return out if keep else out.squeeze(dim=axes)
    wide = src.to(acc) if acc != src.dtype else src
    if node.op.name == "sum":
        return wide.sum(dim=axes, keepdim=keep)
    return wide.mean(dim=axes, keepdim=keep)


def evaluate_node(node, args: Sequence[torch.Tensor]) -> torch.Tensor:
    """reference.py:74-112."""
    op = node.op.name
    if op in _UNARY:
        return _UNARY[op](args[0])
    if op in _BINARY:
        return _BINARY[op](args[0], args[1])
    if op == "cast":
        return args[0].to(TORCH[node.output.dtype.name])
    if op == "matmul":
        return args[0] @ args[1]
    if op in ("sum", "mean", "max"):
        return _reduce(node, args[0])
    if op == "reshape":
        return args[0].reshape(tuple(node.attrs["sizes"]))
    if op == "transpose":
        return args[0].permute(tuple(node.attrs["permutation"]))
    if op == "concat":
        return torch.cat([args[0], args[1]], dim=int(node.attrs["axis"]))
    if op == "slice":
        return args[0].narrow(int(node.attrs["axis"]), int(node.attrs["start"]), int(node.attrs["length"])).contiguous()
    if op == "broadcast_to":
        return args[0].broadcast_to(_sizes(node.output)).contiguous()
    if op == "constant":
        return torch.full((), float(node.attrs["value"]), dtype=TORCH[node.output.dtype.name])
    if op in ("print", "assert_finite"):
        return args[0]
    raise NotImplementedError(f"the interpreter does not implement {op}")


def interpret(graph, feeds: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """reference.py:141-165: every intermediate kept; feeds must have the declared dtype."""
    missing = [v.name for v in graph.inputs if v.name not in feeds]
    if missing:
        raise KeyError(f"no value supplied for {missing}")
    env: dict[str, torch.Tensor] = {}
    for v in graph.inputs:
        t = feeds[v.name]
        if t.dtype != TORCH[v.dtype.name]:
            raise TypeError(f"{v.name} was declared {v.dtype.name} and was given {t.dtype}")
        env[v.name] = t
    for n in graph.nodes:
        env[n.output.name] = evaluate_node(n, [env[i] for i in n.inputs])
    return env


def run(graph, feeds: dict[str, torch.Tensor]) -> list[torch.Tensor]:
    env = interpret(graph, feeds)
    return [env[o] for o in graph.outputs]


def random_feeds(graph, *, seed: int = 0, scale: float = 1.0, positive: bool = False) -> dict[str, torch.Tensor]:
    """reference.py:174-205: one seeded generator, inputs in declaration order."""
    g = torch.Generator().manual_seed(seed)
    feeds = {}
    for v in graph.inputs:
        sizes = list(_sizes(v))
        dt = TORCH[v.dtype.name]
        if v.dtype.kind == "float":
            s = torch.randn(sizes, generator=g, dtype=torch.float32) * scale
            if positive:
                s = s.abs() + 0.5
            feeds[v.name] = s.to(dt)
        elif v.dtype.name == "bool":
            feeds[v.name] = torch.randint(0, 2, sizes, generator=g, dtype=torch.int64).to(torch.bool)
        else:
            feeds[v.name] = torch.randint(-4, 5, sizes, generator=g, dtype=torch.int64).to(dt)
    return feeds


def outputs_agree(left, right, *, tolerance: float = 0.0) -> bool:
    """reference.py:208-228: bit equality at tolerance 0, else allclose(atol=rtol=tolerance)."""
    if len(left) != len(right):
        return False
    for a, b in zip(left, right, strict=True):
        a, b = a.cpu(), b.cpu()
        if a.shape != b.shape:
            return False
        if tolerance == 0.0:
            if not torch.equal(a, b):
                return False
        elif not torch.allclose(a.float(), b.float(), atol=tolerance, rtol=tolerance):
            return False
    return True


def largest_difference(left, right) -> float:
    worst = 0.0
    for a, b in zip(left, right, strict=True):
        worst = max(worst, float((a.cpu().float() - b.cpu().float()).abs().max()))
    return worst


def relative_difference(left, right) -> float:
    """reference.py:240-248: worst absolute difference over the largest |value| on the left."""
    scale = max((float(t.cpu().float().abs().max()) for t in left), default=0.0)
    if scale == 0.0:
        return largest_difference(left, right)
    return largest_difference(left, right) / scale


def generated_python_program(graph):
    """tgc's compile path on the CPU: exact pipeline, depth-first order, liveness over nodes,
    largest-first plan, then the arena program (executor.py:91-122). Uses tgcb's restatements
    of tgc's pipeline and planner, which the golden tests pin to tgc's printed graphs."""
    from tgcb import memory, passes

    opt, _ = passes.default_pipeline().run(graph)
    order = memory.depth_first_order(opt)
    sizes = {v.name: v.bytes for v in opt.inputs}
    sizes.update({n.output.name: n.output.bytes for n in opt.nodes})
    steps = [(list(n.inputs), [n.output.name]) for n in order]
    intervals = memory.intervals_for_steps([v.name for v in opt.inputs], steps, list(opt.outputs), sizes)
    plan = memory.plan_largest_first(intervals)
    return ArenaProgram(opt, order, {a.name: a.offset for a in plan.allocations}, plan.arena_bytes)


class ArenaProgram:
    """tgc's generated-Python execution (emit.py:92-209, executor.py:52-79) on the CPU.

    ``plan`` maps value name -> byte offset (tgc's unaligned largest-first plan, element
    offset = byte offset // 4, emit.py:177-196); ``arena_bytes`` its size. Each call zeroes
    a fresh arena like ``CompiledGraph.__call__`` does, copies the inputs into their views,
    runs one torch op per node in ``order`` and returns views of the outputs.
    """

    def __init__(self, graph, order, offsets: dict[str, int], arena_bytes: int):
        self.graph = graph
        self.order = list(order)
        self.offsets = offsets
        self.arena_elements = -(-arena_bytes // 4)
        self.dtype = TORCH[graph.inputs[0].dtype.name]

    def _view(self, arena: torch.Tensor, value) -> torch.Tensor:
        off = self.offsets[value.name] // 4
        sizes = _sizes(value)
        n = 1
        for s in sizes:
            n *= s
        return arena[off : off + n].reshape(sizes).view(TORCH[value.dtype.name])

    def __call__(self, feeds: dict[str, torch.Tensor], arena: torch.Tensor | None = None) -> list[torch.Tensor]:
        if arena is None:
            arena = torch.zeros(self.arena_elements, dtype=self.dtype)
        bufs = {}
        for v in self.graph.inputs:
            bufs[v.name] = self._view(arena, v)
            bufs[v.name].copy_(feeds[v.name])
        for n in self.order:
            bufs[n.output.name] = self._view(arena, n.output)
        for n in self.order:
            target = bufs[n.output.name]
            if n.op.name == "constant":
                target.fill_(float(n.attrs["value"]))
            else:
                target.copy_(evaluate_node(n, [bufs[i] for i in n.inputs]))
        return [bufs[o] for o in self.graph.outputs]
