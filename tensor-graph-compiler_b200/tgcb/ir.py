"""The graph IR the backend compiles: element types, the op table, shapes, graphs, a builder.

This is a host-side restatement of tgc's IR so the backend runs where tgc is not installed
(the GPU hosts). Names, attribute keys, promotion, shape inference and error classes follow
tgc so that a graph built here and one built by tgc are interchangeable, and the lowering in
``tgcb.codegen`` only reads the attributes both share (``nodes``, ``inputs``, ``outputs``,
``node.op.name``, ``node.inputs``, ``node.output.{name,shape,dtype}``, ``node.attrs``). That
duck-typed surface is what lets ``tgcb.runtime.compile_graph`` accept tgc's own ``Graph``
objects unchanged.

Reference map:
  DType / promotion / accumulator widening .... tgc/ir/dtype.py:15-151
  Op and the op table ......................... tgc/ir/op.py:30-161
  Dim / Shape / broadcast / matmul / reduce ... tgc/ir/shape.py:21-247
  Value / Node / Graph / validate ............. tgc/ir/graph.py:33-225
  infer_output and per-category rules ......... tgc/ir/graph.py:239-380
  Builder ..................................... tgc/ir/builder.py:21-201
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from dataclasses import dataclass, field

from tgcb.errors import ConfigError, GraphError, TypeInferenceError

# ----------------------------------------------------------------------------- element types


@dataclass(frozen=True)
class DType:
    """One element type: a name, a width in bits and a kind (tgc/ir/dtype.py:15)."""

    name: str
    bits: int
    kind: str

    def __post_init__(self) -> None:
        if self.bits < 1:
            raise ConfigError(f"{self.name} has no width")
        if self.kind not in ("float", "int", "uint", "bool"):
            raise ConfigError(f"unknown kind {self.kind!r} for {self.name}")

    @property
    def bytes(self) -> int:
        return max(1, self.bits // 8)

    @property
    def is_float(self) -> bool:
        return self.kind == "float"

    @property
    def is_integral(self) -> bool:
        return self.kind in ("int", "uint", "bool")

    def __str__(self) -> str:
        return self.name


BOOL = DType("bool", 8, "bool")
INT8 = DType("int8", 8, "int")
INT32 = DType("int32", 32, "int")
INT64 = DType("int64", 64, "int")
FLOAT16 = DType("float16", 16, "float")
BFLOAT16 = DType("bfloat16", 16, "float")
FLOAT32 = DType("float32", 32, "float")
FLOAT64 = DType("float64", 64, "float")

ALL_DTYPES = (BOOL, INT8, INT32, INT64, FLOAT16, BFLOAT16, FLOAT32, FLOAT64)
DTYPES_BY_NAME = {d.name: d for d in ALL_DTYPES}
_FLOAT_LADDER = (FLOAT16, BFLOAT16, FLOAT32, FLOAT64)
_INT_LADDER = (BOOL, INT8, INT32, INT64)


def dtype_from_name(name: str) -> DType:
    """Look a type up by name (tgc/ir/dtype.py:61)."""
    try:
        return DTYPES_BY_NAME[name]
    except KeyError:
        raise ConfigError(f"unknown dtype {name!r}, expected one of {sorted(DTYPES_BY_NAME)}") from None


def promote(left: DType, right: DType) -> DType:
    """Result type of a binary op: float beats int, wider beats narrower (tgc/ir/dtype.py:68-86)."""
    if left == right:
        return left
    if left.is_float and right.is_float:
        if {left, right} == {FLOAT16, BFLOAT16}:
            raise TypeInferenceError(
                "float16 and bfloat16 have the same width and neither contains the other, "
                "so the graph has to say which it wants"
            )
        return max(left, right, key=_FLOAT_LADDER.index)
    if left.is_float:
        return left
    if right.is_float:
        return right
    for d in (left, right):
        if d not in _INT_LADDER:
            raise TypeInferenceError(f"no promotion rule for {d}")
    return max(left, right, key=_INT_LADDER.index)


def promote_all(dtypes: Sequence[DType]) -> DType:
    if not dtypes:
        raise TypeInferenceError("there is nothing to promote")
    out = dtypes[0]
    for d in dtypes[1:]:
        out = promote(out, d)
    return out


def accumulator_for(dtype: DType) -> DType:
    """Reductions widen narrow floats to float32 and bool/int8 to int32 (tgc/ir/dtype.py:139-151)."""
    if dtype in (FLOAT16, BFLOAT16):
        return FLOAT32
    if dtype in (BOOL, INT8):
        return INT32
    return dtype


def can_represent_exactly(dtype: DType, value: int) -> bool:
    """Whether an integer survives a round trip through ``dtype`` (tgc/ir/dtype.py:121-136)."""
    if dtype.is_integral:
        if dtype is BOOL:
            return value in (0, 1)
        half = 2 ** (dtype.bits - 1)
        return -half <= value < half
    mantissa = {FLOAT16: 11, BFLOAT16: 8, FLOAT32: 24, FLOAT64: 53}[dtype]
    return abs(value) <= 2**mantissa


# ----------------------------------------------------------------------------- operations

ELEMENTWISE = "elementwise"
REDUCTION = "reduction"
CONTRACTION = "contraction"
VIEW = "view"
LEAF = "leaf"
SIDE_EFFECT = "side_effect"
CATEGORIES = (ELEMENTWISE, REDUCTION, CONTRACTION, VIEW, LEAF, SIDE_EFFECT)


@dataclass(frozen=True)
class Op:
    """An operation and the properties passes ask about (tgc/ir/op.py:30-80)."""

    name: str
    category: str
    arity: int = 1
    commutative: bool = False
    pure: bool = True
    reads_input_once: bool = True
    identity_element: float | None = None

    def __post_init__(self) -> None:
        if not self.name:
            raise ConfigError("an op needs a name")
        if self.category not in CATEGORIES:
            raise ConfigError(f"unknown category {self.category!r} for {self.name}")
        if self.arity < 0:
            raise ConfigError(f"{self.name} cannot take {self.arity} inputs")
        if self.commutative and self.arity != 2:
            raise ConfigError(f"{self.name} is commutative but takes {self.arity} inputs")

    @property
    def is_elementwise(self) -> bool:
        return self.category == ELEMENTWISE

    @property
    def is_leaf(self) -> bool:
        return self.category == LEAF

    @property
    def can_be_removed_if_unused(self) -> bool:
        return self.pure and self.category != SIDE_EFFECT

    def __str__(self) -> str:
        return self.name


ADD = Op("add", ELEMENTWISE, 2, commutative=True, identity_element=0.0)
MUL = Op("mul", ELEMENTWISE, 2, commutative=True, identity_element=1.0)
SUB = Op("sub", ELEMENTWISE, 2)
DIV = Op("div", ELEMENTWISE, 2)
MAXIMUM = Op("maximum", ELEMENTWISE, 2, commutative=True)
MINIMUM = Op("minimum", ELEMENTWISE, 2, commutative=True)
NEG = Op("neg", ELEMENTWISE)
EXP = Op("exp", ELEMENTWISE)
LOG = Op("log", ELEMENTWISE)
SQRT = Op("sqrt", ELEMENTWISE)
TANH = Op("tanh", ELEMENTWISE)
RELU = Op("relu", ELEMENTWISE)
SIGMOID = Op("sigmoid", ELEMENTWISE)
RECIPROCAL = Op("reciprocal", ELEMENTWISE)
ABS = Op("abs", ELEMENTWISE)
CAST = Op("cast", ELEMENTWISE)
STEP = Op("step", ELEMENTWISE)
SUM = Op("sum", REDUCTION)
MAX = Op("max", REDUCTION)
MEAN = Op("mean", REDUCTION)
MATMUL = Op("matmul", CONTRACTION, 2)
CONCAT = Op("concat", VIEW, 2)
SLICE = Op("slice", VIEW)
RESHAPE = Op("reshape", VIEW)
TRANSPOSE = Op("transpose", VIEW)
BROADCAST_TO = Op("broadcast_to", VIEW)
INPUT = Op("input", LEAF, 0)
CONSTANT = Op("constant", LEAF, 0)
PRINT = Op("print", SIDE_EFFECT, pure=False)
ASSERT_FINITE = Op("assert_finite", SIDE_EFFECT, pure=False)

ALL_OPS = (
    ADD, MUL, SUB, DIV, MAXIMUM, MINIMUM, NEG, EXP, LOG, SQRT, TANH, RELU, SIGMOID,
    RECIPROCAL, ABS, CAST, STEP, SUM, MAX, MEAN, MATMUL, RESHAPE, TRANSPOSE, BROADCAST_TO,
    CONCAT, SLICE, INPUT, CONSTANT, PRINT, ASSERT_FINITE,
)
OPS_BY_NAME = {o.name: o for o in ALL_OPS}


def get_op(name: str) -> Op:
    try:
        return OPS_BY_NAME[name]
    except KeyError:
        raise ConfigError(f"unknown op {name!r}") from None


# ----------------------------------------------------------------------------- shapes


@dataclass(frozen=True)
class Dim:
    """A dimension: a known size or a symbolic name (tgc/ir/shape.py:21-50)."""

    value: int | None = None
    name: str = ""

    def __post_init__(self) -> None:
        if self.value is None and not self.name:
            raise ConfigError("a dimension is either a size or a name")
        if self.value is not None and self.value < 0:
            raise ConfigError(f"a dimension cannot be negative, got {self.value}")
        if self.value is not None and self.name:
            raise ConfigError("a dimension cannot be both a size and a name")

    @property
    def is_static(self) -> bool:
        return self.value is not None

    @property
    def is_one(self) -> bool:
        return self.value == 1

    def __str__(self) -> str:
        return str(self.value) if self.is_static else self.name


def dim(size: int | str) -> Dim:
    return Dim(name=size) if isinstance(size, str) else Dim(value=int(size))


@dataclass(frozen=True)
class Shape:
    """The dimensions of a tensor (tgc/ir/shape.py:62-108)."""

    sizes: tuple[Dim, ...] = ()

    @property
    def rank(self) -> int:
        return len(self.sizes)

    @property
    def is_static(self) -> bool:
        return all(s.is_static for s in self.sizes)

    @property
    def elements(self) -> int:
        if not self.is_static:
            raise TypeInferenceError(f"the size of {self} is not known until it runs")
        n = 1
        for s in self.sizes:
            n *= s.value or 0
        return n

    def bytes_for(self, element_size: int) -> int:
        if element_size < 1:
            raise ConfigError("an element takes at least one byte")
        return self.elements * element_size

    def ints(self) -> tuple[int, ...]:
        """The sizes as plain integers; refuses symbolic dimensions."""
        if not self.is_static:
            raise TypeInferenceError(f"{self} has a symbolic dimension")
        return tuple(s.value or 0 for s in self.sizes)

    def __str__(self) -> str:
        return "[" + ", ".join(str(s) for s in self.sizes) + "]"

    def __len__(self) -> int:
        return len(self.sizes)

    def __getitem__(self, index: int) -> Dim:
        return self.sizes[index]


def shape(*sizes: int | str) -> Shape:
    return Shape(tuple(dim(s) for s in sizes))


def dims_equal(a: Dim, b: Dim) -> bool:
    """Certainly equal: both static and equal, or the same symbol (tgc/ir/shape.py:112-124)."""
    if a.is_static and b.is_static:
        return a.value == b.value
    if a.is_static or b.is_static:
        return False
    return a.name == b.name


def _broadcast_dim(a: Dim, b: Dim) -> Dim:
    if dims_equal(a, b):
        return a
    if a.is_one:
        return b
    if b.is_one:
        return a
    if not (a.is_static and b.is_static):
        raise TypeInferenceError(
            f"cannot broadcast {a} against {b} without knowing whether either is one"
        )
    raise TypeInferenceError(f"cannot broadcast a dimension of {a} against {b}")


def broadcast(left: Shape, right: Shape) -> Shape:
    """Right-aligned broadcasting (tgc/ir/shape.py:141-153)."""
    rank = max(left.rank, right.rank)
    one = Dim(value=1)
    out = []
    for k in range(1, rank + 1):
        a = left.sizes[-k] if k <= left.rank else one
        b = right.sizes[-k] if k <= right.rank else one
        out.append(_broadcast_dim(a, b))
    return Shape(tuple(reversed(out)))


def broadcast_all(shapes: Sequence[Shape]) -> Shape:
    if not shapes:
        raise TypeInferenceError("there is nothing to broadcast")
    out = shapes[0]
    for s in shapes[1:]:
        out = broadcast(out, s)
    return out


def matmul_shape(left: Shape, right: Shape) -> Shape:
    """(..., m, k) @ (..., k, n) with broadcast batch dims (tgc/ir/shape.py:181-190)."""
    if left.rank < 2 or right.rank < 2:
        raise TypeInferenceError(f"a matrix product needs two matrices, got {left} and {right}")
    if not dims_equal(left.sizes[-1], right.sizes[-2]):
        raise TypeInferenceError(
            f"{left} and {right} do not meet: {left.sizes[-1]} against {right.sizes[-2]}"
        )
    batch = broadcast(Shape(left.sizes[:-2]), Shape(right.sizes[:-2]))
    return Shape((*batch.sizes, left.sizes[-2], right.sizes[-1]))


def normalise_axes(axes: Sequence[int], rank: int) -> tuple[int, ...]:
    """Sorted non-negative axes, refusing duplicates and out-of-range (tgc/ir/shape.py:207-219)."""
    if rank < 0:
        raise ConfigError("a rank cannot be negative")
    seen: set[int] = set()
    for a in axes:
        r = a + rank if a < 0 else a
        if not 0 <= r < rank:
            raise ConfigError(f"axis {a} is outside a tensor of rank {rank}")
        if r in seen:
            raise ConfigError(f"axis {a} is given twice")
        seen.add(r)
    return tuple(sorted(seen))


def reduce_shape(source: Shape, axes: Sequence[int], *, keepdims: bool = False) -> Shape:
    axes_n = normalise_axes(axes, source.rank)
    kept = []
    for i, s in enumerate(source.sizes):
        if i in axes_n:
            if keepdims:
                kept.append(Dim(value=1))
            continue
        kept.append(s)
    return Shape(tuple(kept))


def transpose_shape(source: Shape, permutation: Sequence[int]) -> Shape:
    if sorted(permutation) != list(range(source.rank)):
        raise ConfigError(
            f"a permutation of rank {source.rank} must use each axis once, got {list(permutation)}"
        )
    return Shape(tuple(source.sizes[a] for a in permutation))


def reshape_shape(source: Shape, sizes: Sequence[int]) -> Shape:
    """Reshape with at most one ``-1`` (tgc/ir/shape.py:230-253)."""
    inferred = [i for i, s in enumerate(sizes) if s == -1]
    if len(inferred) > 1:
        raise ConfigError("at most one dimension can be inferred")
    if any(s < -1 or s == 0 for s in sizes):
        raise ConfigError(f"a reshape target must be positive or -1, got {list(sizes)}")
    if not inferred:
        target = Shape(tuple(dim(s) for s in sizes))
        if source.is_static and target.elements != source.elements:
            raise TypeInferenceError(f"cannot reshape {source.elements} elements into {target}")
        return target
    known = 1
    for s in sizes:
        if s != -1:
            known *= s
    if source.elements % known != 0:
        raise TypeInferenceError(f"cannot reshape {source} into {list(sizes)}")
    resolved = list(sizes)
    resolved[inferred[0]] = source.elements // known
    return Shape(tuple(dim(s) for s in resolved))


def contiguous_strides(sizes: Sequence[int]) -> tuple[int, ...]:
    """Row-major element strides of a packed tensor."""
    strides = [1] * len(sizes)
    for i in range(len(sizes) - 2, -1, -1):
        strides[i] = strides[i + 1] * sizes[i + 1]
    return tuple(strides)


# ----------------------------------------------------------------------------- graphs


@dataclass(frozen=True)
class Value:
    """One tensor produced by one node (tgc/ir/graph.py:33-50)."""

    name: str
    shape: Shape
    dtype: DType

    def __post_init__(self) -> None:
        if not self.name:
            raise ConfigError("a value needs a name")

    @property
    def bytes(self) -> int:
        return self.shape.bytes_for(self.dtype.bytes)

    def __str__(self) -> str:
        return f"{self.name}: {self.dtype}{self.shape}"


def _hashable(v: object) -> object:
    return tuple(v) if isinstance(v, list) else v


@dataclass
class Node:
    """One operation applied to named values (tgc/ir/graph.py:53-99)."""

    op: Op
    inputs: tuple[str, ...]
    output: Value
    attrs: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.op.arity >= 0 and len(self.inputs) != self.op.arity:
            raise GraphError(f"{self.op} takes {self.op.arity} inputs, got {len(self.inputs)}")

    @property
    def name(self) -> str:
        return self.output.name

    def signature(self) -> tuple:
        """Key shared by nodes computing the same thing; commutative operands sorted."""
        ins = tuple(sorted(self.inputs)) if self.op.commutative else self.inputs
        attrs = tuple(sorted((k, _hashable(v)) for k, v in self.attrs.items()))
        return (self.op.name, ins, attrs, self.output.dtype.name)

    def replace_inputs(self, mapping: dict[str, str]) -> Node:
        return Node(self.op, tuple(mapping.get(n, n) for n in self.inputs), self.output, dict(self.attrs))

    def __str__(self) -> str:
        extra = ""
        if self.attrs:
            extra = " {" + ", ".join(f"{k}={v}" for k, v in sorted(self.attrs.items())) + "}"
        return f"{self.output.name} = {self.op.name}({', '.join(self.inputs)}){extra}"


@dataclass
class Graph:
    """A single-assignment graph, nodes kept in topological order (tgc/ir/graph.py:109-196)."""

    nodes: list[Node] = field(default_factory=list)
    inputs: list[Value] = field(default_factory=list)
    outputs: list[str] = field(default_factory=list)

    def __iter__(self) -> Iterator[Node]:
        return iter(self.nodes)

    def __len__(self) -> int:
        return len(self.nodes)

    @property
    def value_names(self) -> set[str]:
        return {v.name for v in self.inputs} | {n.name for n in self.nodes}

    def value(self, name: str) -> Value:
        for v in self.inputs:
            if v.name == name:
                return v
        for n in self.nodes:
            if n.name == name:
                return n.output
        raise GraphError(f"no value named {name!r}")

    def node(self, name: str) -> Node:
        for n in self.nodes:
            if n.name == name:
                return n
        raise GraphError(f"no node produces {name!r}")

    def producer_of(self, name: str) -> Node | None:
        for n in self.nodes:
            if n.name == name:
                return n
        return None

    def consumers_of(self, name: str) -> list[Node]:
        return [n for n in self.nodes if name in n.inputs]

    def use_counts(self) -> dict[str, int]:
        counts = dict.fromkeys(self.value_names, 0)
        for n in self.nodes:
            for i in n.inputs:
                counts[i] = counts.get(i, 0) + 1
        for o in self.outputs:
            counts[o] = counts.get(o, 0) + 1
        return counts

    def clone(self) -> Graph:
        return Graph(
            [Node(n.op, n.inputs, n.output, dict(n.attrs)) for n in self.nodes],
            list(self.inputs),
            list(self.outputs),
        )

    def with_nodes(self, nodes: Sequence[Node]) -> Graph:
        return Graph(list(nodes), list(self.inputs), list(self.outputs))

    def __str__(self) -> str:
        header = ", ".join(str(v) for v in self.inputs)
        body = "\n".join(f"  {n}" for n in self.nodes)
        return f"graph({header}) {{\n{body}\n  return {', '.join(self.outputs)}\n}}"


def adopt(graph) -> Graph:
    """``graph`` as a tgcb Graph. A tgcb Graph is returned as it is; a graph of tgc's own IR
    (tgc/ir/graph.py:109-196: ``inputs`` of values, ``nodes`` in topological order, ``outputs``
    by name) is rebuilt value by value, looking each operation and dtype up by its name, so
    it prints, validates and compiles exactly like the same graph built with tgcb's Builder."""
    if isinstance(graph, Graph):
        return graph

    def value(v) -> Value:
        dims = tuple(Dim(d.value, d.name) for d in v.shape.sizes)
        return Value(v.name, Shape(dims), dtype_from_name(v.dtype.name))

    try:
        inputs = [value(v) for v in graph.inputs]
        nodes = [Node(get_op(n.op.name), tuple(n.inputs), value(n.output), dict(n.attrs)) for n in graph.nodes]
        outputs = list(graph.outputs)
    except AttributeError as e:
        raise GraphError(f"not a graph: {e}") from None
    return Graph(nodes, inputs, outputs)


def validate(graph) -> None:
    """Topological order, single assignment, defined outputs (tgc/ir/graph.py:199-225)."""
    defined: set[str] = set()
    for v in graph.inputs:
        if v.name in defined:
            raise GraphError(f"input {v.name!r} is declared twice")
        defined.add(v.name)
    for n in graph.nodes:
        for i in n.inputs:
            if i not in defined:
                raise GraphError(
                    f"{n.name} reads {i!r} before it is defined, "
                    "so the node list is not in topological order"
                )
        if n.name in defined:
            raise GraphError(f"{n.name!r} is assigned twice")
        defined.add(n.name)
    if not graph.outputs:
        raise GraphError("a graph with no outputs computes nothing")
    for o in graph.outputs:
        if o not in defined:
            raise GraphError(f"output {o!r} is not defined")


def reachable_from_outputs(graph) -> set[str]:
    """Every value an output depends on (tgc/ir/graph.py:407-419)."""
    wanted = set(graph.outputs)
    changed = True
    while changed:
        changed = False
        for n in reversed(graph.nodes):
            if n.name in wanted:
                for i in n.inputs:
                    if i not in wanted:
                        wanted.add(i)
                        changed = True
    return wanted


_FLOAT_RESULT_OPS = ("exp", "log", "sqrt", "tanh", "sigmoid", "reciprocal", "div")


def infer_output(op: Op, operands: Sequence[Value], attrs: dict, name: str) -> Value:
    """The value an op produces from what it reads (tgc/ir/graph.py:239-380)."""
    if op.category == ELEMENTWISE:
        if not operands:
            raise TypeInferenceError(f"{op} needs at least one input")
        out_shape = broadcast_all([o.shape for o in operands])
        if op is CAST:
            target = attrs.get("dtype")
            if not isinstance(target, DType):
                raise TypeInferenceError("a cast needs a target dtype")
            return Value(name, out_shape, target)
        dt = promote_all([o.dtype for o in operands])
        if op.name in _FLOAT_RESULT_OPS and not dt.is_float:
            dt = FLOAT32
        return Value(name, out_shape, dt)
    if op.category == REDUCTION:
        src = operands[0]
        axes = attrs.get("axes")
        if axes is None:
            raise TypeInferenceError(f"{op} needs axes")
        out_shape = reduce_shape(src.shape, axes, keepdims=bool(attrs.get("keepdims", False)))
        dt = src.dtype if op is MAX else accumulator_for(src.dtype)
        return Value(name, out_shape, dt)
    if op is MATMUL:
        a, b = operands
        return Value(name, matmul_shape(a.shape, b.shape), promote_all([a.dtype, b.dtype]))
    if op.category == VIEW:
        return _infer_view(op, operands, attrs, name)
    if op.category == SIDE_EFFECT:
        return Value(name, operands[0].shape, operands[0].dtype)
    raise TypeInferenceError(f"no inference rule for {op}")


def _infer_view(op: Op, operands: Sequence[Value], attrs: dict, name: str) -> Value:
    src = operands[0]
    if op is RESHAPE:
        sizes = attrs.get("sizes")
        if sizes is None:
            raise TypeInferenceError("a reshape needs target sizes")
        return Value(name, reshape_shape(src.shape, sizes), src.dtype)
    if op is TRANSPOSE:
        perm = attrs.get("permutation")
        if perm is None:
            raise TypeInferenceError("a transpose needs a permutation")
        return Value(name, transpose_shape(src.shape, perm), src.dtype)
    if op is BROADCAST_TO:
        target = attrs.get("shape")
        if not isinstance(target, Shape):
            raise TypeInferenceError("a broadcast needs a target shape")
        return Value(name, broadcast_all([src.shape, target]), src.dtype)
    if op is CONCAT:
        left, right = operands
        axis = attrs.get("axis")
        if axis is None:
            raise TypeInferenceError("a concat needs an axis")
        axis = int(axis)
        if left.shape.rank != right.shape.rank:
            raise TypeInferenceError(f"cannot join rank {left.shape.rank} to rank {right.shape.rank}")
        if not 0 <= axis < left.shape.rank:
            raise TypeInferenceError(f"axis {axis} is outside a rank {left.shape.rank} shape")
        sizes: list[Dim] = []
        for p in range(left.shape.rank):
            a, b = left.shape.sizes[p], right.shape.sizes[p]
            if p == axis:
                sizes.append(dim(a.value + b.value) if a.is_static and b.is_static else dim(f"{a}+{b}"))
                continue
            if not dims_equal(a, b):
                raise TypeInferenceError(
                    f"a join along axis {axis} needs axis {p} to match, got {a} and {b}"
                )
            sizes.append(a)
        return Value(name, Shape(tuple(sizes)), promote_all([left.dtype, right.dtype]))
    if op is SLICE:
        axis, start, length = attrs.get("axis"), attrs.get("start"), attrs.get("length")
        if axis is None or start is None or length is None:
            raise TypeInferenceError("a slice needs an axis, a start and a length")
        axis, start, length = int(axis), int(start), int(length)
        if not 0 <= axis < src.shape.rank:
            raise TypeInferenceError(f"axis {axis} is outside a rank {src.shape.rank} shape")
        if start < 0 or length < 1:
            raise TypeInferenceError(f"a window of {length} at {start} is not a window")
        size = src.shape.sizes[axis]
        if size.is_static and start + length > size.value:
            raise TypeInferenceError(f"a window of {length} at {start} runs off an axis of {size.value}")
        sizes = list(src.shape.sizes)
        sizes[axis] = dim(length)
        return Value(name, Shape(tuple(sizes)), src.dtype)
    raise TypeInferenceError(f"no view rule for {op}")


# ----------------------------------------------------------------------------- builder


@dataclass
class Builder:
    """Accumulates nodes under counter-generated names and returns a validated graph.

    Same method names, argument meaning and naming scheme (``v0``, ``v1``, ...) as
    tgc/ir/builder.py:21-201, so a graph built here prints and serialises like tgc's.
    """

    nodes: list[Node] = field(default_factory=list)
    inputs: list[Value] = field(default_factory=list)
    outputs: list[str] = field(default_factory=list)
    prefix: str = "v"
    _counter: int = field(default=0, repr=False)

    def fresh(self) -> str:
        name = f"{self.prefix}{self._counter}"
        self._counter += 1
        return name

    def _defined(self) -> set[str]:
        return {v.name for v in self.inputs} | {n.name for n in self.nodes}

    def _lookup(self, name: str) -> Value:
        for v in self.inputs:
            if v.name == name:
                return v
        for n in self.nodes:
            if n.name == name:
                return n.output
        raise GraphError(f"no value named {name!r}")

    def input(self, sizes: Sequence[int | str], dtype: DType = FLOAT32, name: str = "") -> str:
        chosen = name or self.fresh()
        if chosen in self._defined():
            raise GraphError(f"{chosen!r} is already defined")
        self.inputs.append(Value(chosen, shape(*sizes), dtype))
        return chosen

    def constant(self, value: float, sizes: Sequence[int | str] = (), dtype: DType = FLOAT32) -> str:
        name = self.fresh()
        out = Value(name, shape(*sizes) if sizes else Shape(), dtype)
        self.nodes.append(Node(CONSTANT, (), out, {"value": float(value)}))
        return name

    def apply(self, op: Op, *names: str, **attrs) -> str:
        operands = [self._lookup(n) for n in names]
        out_name = self.fresh()
        out = infer_output(op, operands, attrs, out_name)
        self.nodes.append(Node(op, tuple(names), out, dict(attrs)))
        return out_name

    def add(self, a: str, b: str) -> str:
        return self.apply(ADD, a, b)

    def sub(self, a: str, b: str) -> str:
        return self.apply(SUB, a, b)

    def mul(self, a: str, b: str) -> str:
        return self.apply(MUL, a, b)

    def div(self, a: str, b: str) -> str:
        return self.apply(DIV, a, b)

    def maximum(self, a: str, b: str) -> str:
        return self.apply(MAXIMUM, a, b)

    def minimum(self, a: str, b: str) -> str:
        return self.apply(MINIMUM, a, b)

    def neg(self, a: str) -> str:
        return self.apply(NEG, a)

    def exp(self, a: str) -> str:
        return self.apply(EXP, a)

    def log(self, a: str) -> str:
        return self.apply(LOG, a)

    def sqrt(self, a: str) -> str:
        return self.apply(SQRT, a)

    def tanh(self, a: str) -> str:
        return self.apply(TANH, a)

    def relu(self, a: str) -> str:
        return self.apply(RELU, a)

    def sigmoid(self, a: str) -> str:
        return self.apply(SIGMOID, a)

    def reciprocal(self, a: str) -> str:
        return self.apply(RECIPROCAL, a)

    def abs(self, a: str) -> str:
        return self.apply(ABS, a)

    def step(self, a: str) -> str:
        return self.apply(STEP, a)

    def cast(self, a: str, dtype: DType) -> str:
        return self.apply(CAST, a, dtype=dtype)

    def sum(self, a: str, axes: Sequence[int], *, keepdims: bool = False) -> str:
        return self.apply(SUM, a, axes=tuple(axes), keepdims=keepdims)

    def mean(self, a: str, axes: Sequence[int], *, keepdims: bool = False) -> str:
        return self.apply(MEAN, a, axes=tuple(axes), keepdims=keepdims)

    def max(self, a: str, axes: Sequence[int], *, keepdims: bool = False) -> str:
        return self.apply(MAX, a, axes=tuple(axes), keepdims=keepdims)

    def matmul(self, a: str, b: str) -> str:
        return self.apply(MATMUL, a, b)

    def reshape(self, a: str, sizes: Sequence[int]) -> str:
        return self.apply(RESHAPE, a, sizes=tuple(sizes))

    def transpose(self, a: str, permutation: Sequence[int]) -> str:
        return self.apply(TRANSPOSE, a, permutation=tuple(permutation))

    def broadcast_to(self, a: str, sizes: Sequence[int | str]) -> str:
        return self.apply(BROADCAST_TO, a, shape=shape(*sizes))

    def concat(self, a: str, b: str, axis: int = 0) -> str:
        return self.apply(CONCAT, a, b, axis=int(axis))

    def slice(self, a: str, axis: int, start: int, length: int) -> str:
        return self.apply(SLICE, a, axis=int(axis), start=int(start), length=int(length))

    def emit(self, name: str) -> str:
        if name not in self._defined():
            raise GraphError(f"cannot return {name!r}, which is not defined")
        self.outputs.append(name)
        return name

    def shape_of(self, name: str) -> Shape:
        return self._lookup(name).shape

    def dtype_of(self, name: str) -> DType:
        return self._lookup(name).dtype

    def finish(self, *names: str) -> Graph:
        for n in names:
            self.emit(n)
        g = Graph(list(self.nodes), list(self.inputs), list(self.outputs))
        validate(g)
        return g
