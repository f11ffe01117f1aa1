"""Per-element CUDA expressions for graph values, with view ops folded into index maps.

Every kernel the backend generates computes values *at an index*: a map kernel at each
element of its output, a row kernel at each column of a row, a GEMM epilogue at each
(row, col) of its tile. ``ExprBuilder.value(name, idx)`` returns a C variable holding value
``name`` at multi-index ``idx`` (a tuple of C integer expressions, one per dimension),
emitting the statements that compute it on first use. Statements are memoised on
``(name, idx)``, so within one kernel every value is computed once per index, and a value
read by several consumers at the same index is shared (the CSE tgc's pipeline did at graph
level, repeated at element level).

View operations never move data here: ``broadcast_to`` zeroes an index, ``transpose``
permutes indices, ``reshape`` linearises and delinearises, ``slice`` offsets one index and
``concat`` selects between two clamped reads. Materialised values (graph inputs, GEMM
outputs, reductions produced by an earlier kernel) are loads from their base pointer with
row-major strides.

Arithmetic follows tgc's interpreter (tgc/verify/reference.py:51-112) op by op in the
declared dtype: float32 ops are single IEEE operations (the generated code is compiled with
``-fmad=false`` so no multiply-add contraction changes a rounding), transcendental ops call
CUDA's own ``expf``/``logf``/``tanhf``/``sqrtf`` (never reimplemented), and max/min/relu
propagate NaN like torch does.
"""

from __future__ import annotations

import re

import struct
from collections.abc import Callable, Sequence

from tgcb import ir
from tgcb.errors import CodegenError

CTYPES = {
    "float32": "float",
    "float64": "double",
    "int32": "int",
    "int64": "long long",
    "int8": "signed char",
    "bool": "unsigned char",
}


def ctype(dtype) -> str:
    try:
        return CTYPES[dtype.name]
    except KeyError:
        raise CodegenError(f"the B200 backend has no lowering for {dtype.name} values") from None


def literal(value: float, dtype) -> str:
    """A C literal holding exactly what ``torch.full((), value, dtype)`` holds."""
    name = dtype.name
    if name == "float32":
        try:
            bits = struct.unpack("<I", struct.pack("<f", value))[0]
        except OverflowError:
            bits = 0x7F800000 if value > 0 else 0xFF800000
        return f"__int_as_float(0x{bits:08x})"
    if name == "float64":
        bits = struct.unpack("<Q", struct.pack("<d", value))[0]
        return f"__longlong_as_double(0x{bits:016x}LL)"
    if name in ("int32", "int8"):
        return f"(({ctype(dtype)}){int(value)})"
    if name == "int64":
        return f"((long long){int(value)}LL)"
    if name == "bool":
        return "((unsigned char)1)" if value else "((unsigned char)0)"
    raise CodegenError(f"no literal for {name}")


def _is_int(d) -> bool:
    return d.name in ("int8", "int32", "int64", "bool")


def _wrap(op: str, a: str, b: str, d) -> str:
    """Integer add/sub/mul with two's complement wrap, like torch's integer kernels."""
    u = "unsigned long long" if d.name == "int64" else "unsigned int"
    return f"(({ctype(d)})(({u}){a} {op} ({u}){b}))"


def unary_c(name: str, a: str, src, out, approx: bool = False) -> str:
    t = ctype(out)
    if _is_int(src) and out.is_float:
        a = f"(({t}){a})"
    if approx and t == "float" and name in ("exp", "tanh", "sigmoid"):
        return {"exp": f"__expf({a})", "tanh": f"tgcb_tanh_approx({a})", "sigmoid": f"tgcb_sigmoid_approx({a})"}[name]
    if name == "neg":
        return f"(-{a})" if not _is_int(out) else _wrap("-", "0", a, out)
    if name == "exp":
        return f"expf({a})" if t == "float" else f"exp({a})"
    if name == "log":
        return f"logf({a})" if t == "float" else f"log({a})"
    if name == "sqrt":
        return f"sqrtf({a})" if t == "float" else f"sqrt({a})"
    if name == "tanh":
        return f"tanhf({a})" if t == "float" else f"tanh({a})"
    if name == "relu":
        zero = "0" if _is_int(out) else ("0.0f" if t == "float" else "0.0")
        return f"(({a}) > {zero} || ({a}) != ({a}) ? ({a}) : ({t}){zero})"
    if name == "sigmoid":
        return f"(1.0f / (1.0f + expf(-({a}))))" if t == "float" else f"(1.0 / (1.0 + exp(-({a}))))"
    if name == "reciprocal":
        return f"(({t})1 / ({a}))"
    if name == "abs":
        return f"fabsf({a})" if t == "float" else (f"fabs({a})" if t == "double" else f"(({a}) < 0 ? -({a}) : ({a}))")
    if name == "step":
        return f"(({a}) > 0 ? ({t})1 : ({t})0)"
    raise CodegenError(f"no lowering for {name}")


def binary_c(name: str, a: str, b: str, out) -> str:
    t = ctype(out)
    if _is_int(out):
        if name in ("add", "sub", "mul"):
            return _wrap({"add": "+", "sub": "-", "mul": "*"}[name], a, b, out)
    else:
        a, b = f"(({t}){a})", f"(({t}){b})"
        if name == "add":
            return f"({a} + {b})"
        if name == "sub":
            return f"({a} - {b})"
        if name == "mul":
            return f"({a} * {b})"
        if name == "div":
            return f"({a} / {b})"
    if name == "maximum":
        return f"(({a}) != ({a}) || ({a}) > ({b}) ? ({a}) : ({b}))"
    if name == "minimum":
        return f"(({a}) != ({a}) || ({a}) < ({b}) ? ({a}) : ({b}))"
    raise CodegenError(f"no lowering for {name} on {out.name}")


def cast_c(a: str, src, out) -> str:
    t = ctype(out)
    if out.name == "bool":
        return f"((unsigned char)(({a}) != 0))"
    return f"(({t})({a}))"


def _broadcast_index(idx: Sequence[str], out_sizes: Sequence[int], src_sizes: Sequence[int]) -> tuple[str, ...]:
    """Index into a right-aligned broadcast operand: size-1 dims read index 0."""
    r, rs = len(out_sizes), len(src_sizes)
    out = []
    for k in range(rs):
        o = r - rs + k
        out.append("0" if src_sizes[k] == 1 and out_sizes[o] != 1 else idx[o])
    return tuple(out)


def linearise(idx: Sequence[str], sizes: Sequence[int]) -> str:
    if not sizes:
        return "0"
    terms = []
    stride = 1
    for k in range(len(sizes) - 1, -1, -1):
        if sizes[k] != 1:
            terms.append(idx[k] if stride == 1 else f"({idx[k]})*{stride}LL")
        stride *= sizes[k]
    return "(" + " + ".join(terms) + ")" if terms else "0"


def delinearise(lin: str, sizes: Sequence[int]) -> tuple[str, ...]:
    out = []
    stride = 1
    strides = []
    for k in range(len(sizes) - 1, -1, -1):
        strides.append(stride)
        stride *= sizes[k]
    strides.reverse()
    for k, s in enumerate(sizes):
        if s == 1:
            out.append("0")
        elif k == 0:
            out.append(f"(({lin})/{strides[k]}LL)" if strides[k] != 1 else lin)
        else:
            out.append(f"((({lin})/{strides[k]}LL)%{s}LL)" if strides[k] != 1 else f"(({lin})%{s}LL)")
    return tuple(out)


class ExprBuilder:
    """Emits the statements of one kernel body.

    ``pointer_of(name)`` returns a C expression for the base pointer of a materialised value,
    or None if the value is not materialised (then it must be computable from its producer).
    ``resolve(name, idx)`` lets the kernel substitute a register (a GEMM accumulator, a
    row reduction of the same row) before the generic rules apply.
    """

    def __init__(
        self,
        graph_values: dict,
        producers: dict,
        pointer_of: Callable[[str], str | None],
        resolve: Callable[[str, tuple[str, ...]], str | None] | None = None,
        indent: str = "    ",
        approx: bool = False,
    ):
        self.approx = approx  # hardware-approximate exp/tanh/sigmoid (TF32 GEMM epilogues only)
        self.values = graph_values
        self.producers = producers
        self.pointer_of = pointer_of
        self.resolve = resolve or (lambda n, i: None)
        self.lines: list[str] = []
        self.memo: dict[tuple[str, tuple[str, ...]], str] = {}
        self.counter = 0
        self.indent = indent
        self.loads: set[str] = set()
        # (variable, C type, base pointer expression, element offset expression) per load
        self.load_info: list[tuple[str, str, str, str]] = []

    def fresh(self, stem: str) -> str:
        self.counter += 1
        return f"{stem}_{self.counter}"

    def emit(self, line: str) -> None:
        self.lines.append(self.indent + line)

    def sizes(self, name: str) -> tuple[int, ...]:
        return self.values[name].shape.ints()

    def value(self, name: str, idx: Sequence[str]) -> str:
        idx = tuple(idx)
        key = (name, idx)
        if key in self.memo:
            return self.memo[key]
        out = self._compute(name, idx)
        self.memo[key] = out
        return out

    def _compute(self, name: str, idx: tuple[str, ...]) -> str:
        v = self.values[name]
        t = ctype(v.dtype)
        r = self.resolve(name, idx)
        if r is not None:
            return r
        ptr = self.pointer_of(name)
        if ptr is not None:
            self.loads.add(name)
            var = self.fresh("ld")
            off = linearise(idx, self.sizes(name))
            self.emit(f"const {t} {var} = __ldg(reinterpret_cast<const {t}*>({ptr}) + {off});")
            self.load_info.append((var, t, ptr, off))
            return var
        node = self.producers.get(name)
        if node is None:
            raise CodegenError(f"{name} is neither materialised nor produced by a node")
        op = node.op.name
        if op == "constant":
            return literal(float(node.attrs["value"]), v.dtype)
        if op in ("print", "assert_finite"):
            return self.value(node.inputs[0], idx)
        out_sizes = self.sizes(name)
        if node.op.category == ir.ELEMENTWISE:
            args = []
            for i in node.inputs:
                args.append(self.value(i, _broadcast_index(idx, out_sizes, self.sizes(i))))
            srcs = [self.values[i].dtype for i in node.inputs]
            if op == "cast":
                expr = cast_c(args[0], srcs[0], v.dtype)
            elif len(args) == 1:
                expr = unary_c(op, args[0], srcs[0], v.dtype, self.approx)
            else:
                a, b = args
                if _is_int(v.dtype) is False and any(_is_int(s) for s in srcs):
                    a, b = f"(({t}){a})", f"(({t}){b})"
                expr = binary_c(op, a, b, v.dtype)
            var = self.fresh("e")
            self.emit(f"const {t} {var} = {expr};")
            return var
        if op == "broadcast_to":
            src = node.inputs[0]
            return self.value(src, _broadcast_index(idx, out_sizes, self.sizes(src)))
        if op == "transpose":
            perm = tuple(node.attrs["permutation"])
            src_idx = [""] * len(perm)
            for k, p in enumerate(perm):
                src_idx[p] = idx[k]
            return self.value(node.inputs[0], tuple(src_idx))
        if op == "reshape":
            src = node.inputs[0]
            ss = self.sizes(src)
            if tuple(ss) == tuple(out_sizes):
                return self.value(src, idx)
            squeezed_out = [(i, s) for i, s in zip(idx, out_sizes, strict=True) if s != 1]
            squeezed_src = [s for s in ss if s != 1]
            if [s for _, s in squeezed_out] == squeezed_src:
                it = iter(i for i, _ in squeezed_out)
                return self.value(src, tuple("0" if s == 1 else next(it) for s in ss))
            return self.value(src, delinearise(linearise(idx, out_sizes), ss))
        if op == "slice":
            axis, start = int(node.attrs["axis"]), int(node.attrs["start"])
            src_idx = list(idx)
            src_idx[axis] = f"(({idx[axis]}) + {start})"
            return self.value(node.inputs[0], tuple(src_idx))
        if op == "concat":
            axis = int(node.attrs["axis"])
            left, right = node.inputs
            n_left = self.sizes(left)[axis]
            n_right = self.sizes(right)[axis]
            li = list(idx)
            ri = list(idx)
            li[axis] = f"tgcb_min_ll((long long)({idx[axis]}), {n_left - 1}LL)"
            ri[axis] = f"tgcb_max_ll((long long)({idx[axis]}) - {n_left}LL, 0LL)"
            ri[axis] = f"tgcb_min_ll({ri[axis]}, {n_right - 1}LL)"
            a = self.value(left, tuple(li))
            b = self.value(right, tuple(ri))
            var = self.fresh("cat")
            self.emit(f"const {t} {var} = (({idx[axis]}) < {n_left}) ? ({t}){a} : ({t}){b};")
            return var
        raise CodegenError(
            f"{name} ({op}) has to be materialised by its own kernel before another kernel reads it"
        )


_MUL_PREFIX = "(((float)"


def _split_binary(expr: str) -> tuple[str, str, str] | None:
    """(a, op, b) of a float binary_c expression ``(((float)a) op ((float)b))``, else None."""
    if not (expr.startswith(_MUL_PREFIX) and expr.endswith("))")):
        return None
    inner = expr[len(_MUL_PREFIX):-2]
    for op in ("*", "+", "-"):
        sep = f") {op} ((float)"
        if inner.count(sep) == 1:
            a, b = inner.split(sep)
            return a, op, b
    return None


_DEF = re.compile(r"^(\s*)const float (e_\d+) = (.*);$")


def contract_fma(lines: list[str], finals: Sequence[str]) -> list[str]:
    """Fuse a float product used once, by an add or subtract, into one fmaf (single rounding).

    For TF32 GEMM epilogues only, whose results are compared at TF32 tolerance; everywhere else
    each operation rounds on its own, as the reference's per-operation execution does.
    """
    uses: dict[str, int] = {}
    for text in list(lines) + list(finals):
        for name in re.findall(r"\be_\d+\b", text):
            uses[name] = uses.get(name, 0) + 1
    products: dict[str, tuple[str, str]] = {}
    for line in lines:
        m = _DEF.match(line)
        if m:
            parts = _split_binary(m.group(3))
            if parts and parts[1] == "*":
                products[m.group(2)] = (parts[0], parts[2])
    fused: set[str] = set()
    out = []
    for line in lines:
        m = _DEF.match(line)
        parts = _split_binary(m.group(3)) if m else None
        if parts and parts[1] in "+-":
            a, op, b = parts
            # uses[] counts the definition too: a product read once appears twice
            if a in products and uses.get(a) == 2 and a not in fused:
                pa, pb = products[a]
                c = f"((float){b})" if op == "+" else f"(-((float){b}))"
                fused.add(a)
                line = f"{m.group(1)}const float {m.group(2)} = __fmaf_rn((float){pa}, (float){pb}, {c});"
            elif b in products and uses.get(b) == 2 and b not in fused:
                pa, pb = products[b]
                pa = pa if op == "+" else f"(-((float){pa}))"
                fused.add(b)
                line = f"{m.group(1)}const float {m.group(2)} = __fmaf_rn((float){pa}, (float){pb}, ((float){a}));"
        out.append(line)
    return [ln for ln in out if not ((m := _DEF.match(ln)) and m.group(2) in fused)]
