"""tgc's text format for graphs, read and written.

The format is the one ``tgc.ir.serialize.dumps`` prints (tgc/ir/serialize.py:101-125): a
``graph(name: dtype[dims], ...) {`` header, one ``name: dtype[dims] = op(args) {k=v, ...}``
line per node, and ``return a, b``. Reading it lets the backend compile a graph that tgc
built and printed (a gradient graph from tgc/grad, a fuzzer counterexample) on a host where
tgc is not installed; the round trip is pinned against tgc's printer by the golden tests.
"""

from __future__ import annotations

import re

from tgcb import ir
from tgcb.errors import ParseError

_HEADER = re.compile(r"^graph\((.*)\)\s*\{$")
_INPUT = re.compile(r"^\s*(\w+):\s*(\w+)\[([^\]]*)\]\s*$")
_RETURN = re.compile(r"^\s*return\s+(.*)$")
_ASSIGN = re.compile(r"^\s*(\w+):\s*(\w+)\[([^\]]*)\]\s*=\s*(\w+)\(([^)]*)\)\s*(?:\{(.*)\})?\s*$")


def _fmt_shape(s: ir.Shape) -> str:
    return ", ".join(str(d) for d in s.sizes)


def _fmt_value(v: object) -> str:
    if isinstance(v, ir.DType):
        return f"dtype:{v.name}"
    if isinstance(v, ir.Shape):
        return f"shape:[{_fmt_shape(v)}]"
    if isinstance(v, tuple | list):
        return "[" + ",".join(_fmt_value(x) for x in v) + "]"
    if isinstance(v, bool):
        return "true" if v else "false"
    return str(v)


def dumps(graph) -> str:
    lines = [
        "graph("
        + ", ".join(f"{v.name}: {v.dtype.name}[{_fmt_shape(v.shape)}]" for v in graph.inputs)
        + ") {"
    ]
    for n in graph.nodes:
        attrs = ""
        if n.attrs:
            attrs = " {" + ", ".join(f"{k}={_fmt_value(n.attrs[k])}" for k in sorted(n.attrs)) + "}"
        lines.append(
            f"  {n.name}: {n.output.dtype.name}[{_fmt_shape(n.output.shape)}] = "
            f"{n.op.name}({', '.join(n.inputs)}){attrs}"
        )
    lines.append(f"  return {', '.join(graph.outputs)}")
    lines.append("}")
    return "\n".join(lines) + "\n"


def _parse_shape(text: str) -> ir.Shape:
    t = text.strip()
    if not t:
        return ir.Shape()
    out = []
    for piece in t.split(","):
        tok = piece.strip()
        if not tok:
            raise ParseError(f"an empty dimension in {text!r}")
        out.append(ir.dim(int(tok)) if tok.isdigit() else ir.dim(tok))
    return ir.Shape(tuple(out))


def _split_top(text: str) -> list[str]:
    pieces, depth, cur = [], 0, []
    for ch in text:
        if ch in "[(":
            depth += 1
        elif ch in "])":
            depth -= 1
        if ch == "," and depth == 0:
            pieces.append("".join(cur).strip())
            cur = []
            continue
        cur.append(ch)
    if cur:
        pieces.append("".join(cur).strip())
    return [p for p in pieces if p]


def _parse_value(text: str) -> object:
    t = text.strip()
    if t in ("true", "false"):
        return t == "true"
    if t.startswith("dtype:"):
        return ir.dtype_from_name(t[6:])
    if t.startswith("shape:["):
        return _parse_shape(t[7:-1])
    if t.startswith("[") and t.endswith("]"):
        inner = t[1:-1].strip()
        return tuple(_parse_value(p) for p in inner.split(",")) if inner else ()
    try:
        return int(t)
    except ValueError:
        pass
    try:
        return float(t)
    except ValueError:
        return t


def loads(text: str) -> ir.Graph:
    lines = [ln for ln in text.splitlines() if ln.strip()]
    if not lines:
        raise ParseError("there is nothing to parse")
    head = _HEADER.match(lines[0].strip())
    if head is None:
        raise ParseError(f"the first line is not a graph header: {lines[0]!r}")
    inputs = []
    if head.group(1).strip():
        for piece in _split_top(head.group(1).strip()):
            m = _INPUT.match(piece)
            if m is None:
                raise ParseError(f"cannot read the input declaration {piece!r}")
            inputs.append(ir.Value(m.group(1), _parse_shape(m.group(3)), ir.dtype_from_name(m.group(2))))
    nodes, outputs = [], []
    for line in lines[1:]:
        s = line.strip()
        if s == "}":
            continue
        r = _RETURN.match(s)
        if r is not None:
            outputs = [x.strip() for x in r.group(1).split(",") if x.strip()]
            continue
        m = _ASSIGN.match(s)
        if m is None:
            raise ParseError(f"cannot read the assignment {s!r}")
        name, dt, shp, opname, args, attr_text = m.groups()
        attrs: dict = {}
        for piece in _split_top(attr_text or ""):
            if "=" not in piece:
                raise ParseError(f"cannot read the attribute {piece!r}")
            k, _, v = piece.partition("=")
            attrs[k.strip()] = _parse_value(v)
        nodes.append(
            ir.Node(
                ir.get_op(opname),
                tuple(a.strip() for a in args.split(",") if a.strip()),
                ir.Value(name, _parse_shape(shp), ir.dtype_from_name(dt)),
                attrs,
            )
        )
    g = ir.Graph(nodes, inputs, outputs)
    ir.validate(g)
    return g
