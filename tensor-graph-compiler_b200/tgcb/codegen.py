"""Lowering a scheduled graph to B200 kernel steps.

This replaces tgc/codegen/emit.py:165-209. Where tgc writes one torch statement per node
into arena views, this module partitions the graph into kernels and writes each kernel's
CUDA source, which ``tgcb.runtime`` compiles with NVRTC for sm_100a and launches from the
C library.

Partitioning (the grouping tgc's passes/fusion.py and schedule/fusion_search.py reason
about, made executable):

* *Hard* values are graph inputs, ``matmul`` outputs and reduction outputs. Everything else
  (elementwise ops, views, constants) is *soft*: it is recomputed inside whichever kernel
  reads it and never touches HBM unless something forces it to.
* Each ``matmul`` is one GEMM step (tcgen05 TF32 for float32, tcgen05 INT8 with an int32
  accumulator when both operands are int8 values cast to int32). ``transpose`` and the
  int8->int32 ``cast`` on an operand are absorbed into the operand's major-ness and type.
* Reductions over the last axis that share a row space form one *row* step: a multi-phase
  kernel that keeps one row per CTA, computes every reduction of a phase in one pass over
  the row, and feeds them to the next phase (softmax, layernorm, the three-reduction cone).
  Reductions over axis 0 of a matrix are *column* steps, over all axes *full* steps; other
  axis sets fall back to a one-thread-per-output sequential kernel.
* A soft value that must exist in memory (a graph output, or a GEMM operand) is a
  *request*. It is written by the kernel that produces its latest hard dependency if it can
  be computed there: a GEMM epilogue (bias, GELU, loss gradients), or a row step's final
  phase (the normalised layernorm output). Otherwise it gets a standalone elementwise
  *map* step right after its dependencies.
* A hard value read by any kernel other than its producer is stored by its producer.

Reductions declare their bracketing (the order additions happen in) and ``oracle/`` holds
a CPU restatement of each one so reduction results can be checked bit-for-bit when the
summands are exact; against tgc's interpreter (whose ATen order is unspecified) they are
checked within a tolerance.
"""

from __future__ import annotations

import math
import re
from dataclasses import dataclass, field

from tgcb import ir
from tgcb.errors import CodegenError
from tgcb.expr import ExprBuilder, _broadcast_index, contract_fma, ctype, delinearise

NUM_SMS = 148
PAIR_GEMM = True  # whole 256 x 256 tiles run on SM pairs
CHAIN_GEMM = True  # two consecutive SM-pair GEMMs, the second reading the first's rows, share one launch
ROW_PROLOGUE = True  # a one-warp-per-row step producing a chain's first A operand runs inside the chain
# ... when each CTA's epilogue warps have at most this many row groups (16 rows each) to compute
# before their first tile: the MLP block's 8192 rows are 4 rounds over 148 CTAs and gain 2.7%; the
# training step's 65536 rows (28 rounds) kept the epilogue from its first accumulators and lost 0.8%
ROW_PROLOGUE_MAX_ROUNDS = 4
CHAIN_MAX_ITEMS = 32768  # tiles of both GEMMs together (the schedule is a __constant__ table)
K_SPLIT = True  # an SM-pair GEMM with fewer output tiles than pairs cuts K into slices
CHUNKED_MN = True  # tf32 MN-major operands load a stage of 32-column chunks as one 3-D copy
SPLIT_MAX = 8
SPLIT_MIN_KBLOCKS = 16
_LOAD_LINE = re.compile(r"^\s*const (.+?) (ld_\d+) = (.*);$")
_LOAD_NAME = re.compile(r"\b(ld_\d+)\b")
GEMM_THREADS = 576  # tgcb_gemm::THREADS: TMA warp, MMA warp, 16 epilogue warps
CHAIN_THREADS = GEMM_THREADS + 32  # tgcb_gemm::CHAIN_THREADS: plus the warp that publishes stored rows

# Placeholder for the base pointer of a materialised value; replaced once the plan exists.
def PTR(name: str) -> str:
    return f"@P<{name}>@"


@dataclass
class GemmOperand:
    value: str  # materialised 2-D value, row-major storage
    rows: int  # storage rows
    cols: int  # storage cols
    mn_major: bool  # True when the M (or N) index runs along the contiguous storage axis
    elem_bytes: int


@dataclass
class Launch:
    kernel: str
    grid: tuple[int, int, int]
    block: tuple[int, int, int]
    smem: int = 0
    gemm: tuple[GemmOperand, GemmOperand] | None = None
    pair: bool = False  # two-SM GEMM: launched as clusters of two CTAs
    # a chain of two SM-pair GEMMs in one launch: the second GEMM's operands, and the arena
    # value holding its per-row-block counters (zeroed before every launch)
    gemm2: tuple[GemmOperand, GemmOperand] | None = None
    counters: str | None = None
    counter_bytes: int = 0


@dataclass
class Step:
    kind: str
    label: str
    reads: list[str] = field(default_factory=list)
    writes: list[str] = field(default_factory=list)
    source: str = ""
    launches: list[Launch] = field(default_factory=list)
    bracketing: str = ""
    nodes: list[str] = field(default_factory=list)
    pair_gemm: PairGemmInfo | None = None  # set on an SM-pair GEMM step (chain fusion reads it)
    row_body: RowBody | None = None  # set on a one-warp-per-row step (row prologue fusion reads it)


@dataclass
class RowBody:
    """A row step's per-row code for 32 threads (``row``, ``tid``, ``live`` in scope)."""

    lines: str
    nred: int
    rows: int
    cols: int


@dataclass
class PairGemmInfo:
    """What chain fusion needs from an SM-pair GEMM step."""

    M: int
    N: int
    K: int
    is_int: bool
    opa: GemmOperand
    opb: GemmOperand
    epi_name: str
    epi_source: str
    split_scratch: tuple[str, ...] = ()  # the K split's workspace and counters (dropped in a chain)


@dataclass
class RowGroup:
    members: list[str]
    src_sizes: tuple[int, ...]
    phase: dict[str, int] = field(default_factory=dict)


def col_split(rows: int, cols: int) -> tuple[int, int]:
    """(parts, rows per part) of a column reduction over [rows, cols]: enough row blocks for about
    eight CTAs of 256 columns per SM, at least 16 rows each. The parts are [k L, (k + 1) L), so the
    order is tgc's split_sum(column, parts) (tgc/passes/reduction.py:105-121): ceil(rows / parts)
    is L again for every L of this form."""
    cblocks = (cols + 255) // 256
    parts = max(1, min((rows + 15) // 16, (NUM_SMS * 8 + cblocks - 1) // cblocks))
    per = (rows + parts - 1) // parts
    return (rows + per - 1) // per, per


def _prod(xs) -> int:
    p = 1
    for x in xs:
        p *= x
    return p


def _next_pow2(x: int) -> int:
    return 1 << max(0, (x - 1).bit_length())


def row_threads(cols: int, rows: int | None = None) -> int:
    """Threads per row in a row kernel: a power of two in [32, 256] giving each thread at most
    32 columns (a single warp per row up to 1024 columns), so a thread keeps up to 32
    independent loads in flight and reductions of short rows need no block barrier. When there
    are too few rows to give every SM 32 warps, rows get more threads (down to 8 columns per
    thread) so the work spreads evenly over the GPU."""
    t = max(32, min(256, _next_pow2(max(1, (cols + 31) // 32))))
    if rows is not None:
        while t < 256 and rows * (t // 32) < NUM_SMS * 32 and cols >= 16 * t:
            t *= 2
    return t


ROW_BLOCK = 256  # threads per CTA of a row kernel; 256 // T rows are processed side by side
# a standalone row kernel issues all of its first phase's loads before any arithmetic, so each
# thread has its whole row slice in flight at once (the order of the additions is unchanged)
ROW_HOIST_LOADS = True


class Lowering:
    """Partition ``graph`` (already optimised, nodes in ``order``) into kernel steps."""

    def __init__(self, graph, order):
        self.graph = graph
        self.order = list(order)
        self.values = {v.name: v for v in graph.inputs}
        self.values.update({n.name: n.output for n in graph.nodes})
        self.producers = {n.name: n for n in graph.nodes}
        self.inputs = [v.name for v in graph.inputs]
        self.outputs = list(graph.outputs)
        for name, v in self.values.items():
            if not v.shape.is_static:
                raise CodegenError("a symbolic shape cannot be given a fixed offset in an arena")
            ctype(v.dtype)
        self._deps: dict[str, frozenset[str]] = {}
        self.materialised: set[str] = set()  # hard values some other kernel reads
        self.requests: dict[str, str] = {}  # soft value -> owner key
        self.steps: list[Step] = []
        self.scratch: dict[str, int] = {}  # scratch slot name -> bytes
        self.kernel_count = 0
        self.request_pos: dict[str, int] = {}  # soft value written to memory -> emitting step
        self._gen_pos = 0
        self._step_reads: set[str] = set()
        self._frontier_memo: dict = {}

    # ------------------------------------------------------------------ classification

    def is_hard(self, name: str) -> bool:
        node = self.producers.get(name)
        if node is None:
            return True
        return node.op.category in (ir.REDUCTION, ir.CONTRACTION)

    def hard_deps(self, name: str) -> frozenset[str]:
        """Hard values reachable from ``name`` through soft nodes (itself if hard)."""
        if name in self._deps:
            return self._deps[name]
        if self.is_hard(name):
            out = frozenset([name])
        else:
            acc: set[str] = set()
            for i in self.producers[name].inputs:
                acc |= self.hard_deps(i)
            out = frozenset(acc)
        self._deps[name] = out
        return out

    def sizes(self, name: str) -> tuple[int, ...]:
        return self.values[name].shape.ints()

    def reduction_kind(self, node) -> str:
        src = self.sizes(node.inputs[0])
        axes = ir.normalise_axes(node.attrs["axes"], len(src))
        if len(src) >= 1 and axes == (len(src) - 1,):
            return "row"
        if len(src) == 2 and axes == (0,):
            return "col"
        if axes == tuple(range(len(src))):
            return "full"
        return "naive"

    # ------------------------------------------------------------------ gemm operands

    def gemm_operand(self, name: str, want_int8: bool) -> tuple[str, bool, bool]:
        """Peel transposes / no-op reshapes / int8->int32 casts: (base, flipped, from_int8)."""
        cur, flipped, from_int8 = name, False, False
        while True:
            node = self.producers.get(cur)
            if node is None:
                break
            op = node.op.name
            if op == "transpose" and tuple(node.attrs["permutation"]) == (1, 0):
                flipped = not flipped
                cur = node.inputs[0]
                continue
            if op == "reshape" and self.sizes(node.inputs[0]) == self.sizes(cur):
                cur = node.inputs[0]
                continue
            if op in ("print", "assert_finite"):
                cur = node.inputs[0]
                continue
            if (
                want_int8
                and op == "cast"
                and node.output.dtype.name == "int32"
                and self.values[node.inputs[0]].dtype.name == "int8"
            ):
                from_int8 = True
                cur = node.inputs[0]
                continue
            break
        return cur, flipped, from_int8

    # ------------------------------------------------------------------ partition

    def partition(self) -> list[Step]:
        produced_at: dict[str, int] = {n: -1 for n in self.inputs}
        open_groups: dict[tuple[int, ...], RowGroup] = {}
        raw: list[tuple[str, object]] = []  # ("gemm", node) | ("row", group) | ("red", node)

        def close_all():
            for g in list(open_groups.values()):
                raw.append(("row", g))
                for m in g.members:
                    produced_at[m] = len(raw) - 1
            open_groups.clear()

        for node in self.order:
            cat = node.op.category
            if cat == ir.CONTRACTION:
                close_all()
                raw.append(("gemm", node))
                produced_at[node.name] = len(raw) - 1
            elif cat == ir.REDUCTION:
                kind = self.reduction_kind(node)
                if kind != "row":
                    close_all()
                    raw.append(("red", node))
                    produced_at[node.name] = len(raw) - 1
                    continue
                src = node.inputs[0]
                ss = self.sizes(src)
                deps = self.hard_deps(src)
                g = open_groups.get(ss)
                if g is not None:
                    outside = [d for d in deps if d not in g.members]
                    ready = all(d in produced_at for d in outside)
                    aligned = self._row_aligned(node, g)
                    if ready and aligned:
                        inner = [d for d in deps if d in g.members]
                        g.phase[node.name] = 1 + max((g.phase[d] for d in inner), default=0)
                        g.members.append(node.name)
                        continue
                    raw.append(("row", g))
                    for m in g.members:
                        produced_at[m] = len(raw) - 1
                    del open_groups[ss]
                if not all(d in produced_at for d in deps):
                    close_all()
                g = RowGroup([node.name], ss, {node.name: 1})
                open_groups[ss] = g
        close_all()
        self.raw = raw
        self.produced_at = produced_at
        return self._build_steps()

    def _row_aligned(self, node, group: RowGroup) -> bool:
        """Whether ``node``'s source reads group members only at the current row."""
        members = set(group.members)
        ok = True
        R = _prod(group.src_sizes[:-1])
        row_idx = self._row_index(group.src_sizes)

        def resolve(name, idx):
            nonlocal ok
            if name in members:
                if tuple(idx) != self._reduced_row_index(name, row_idx):
                    ok = False
                return "0"
            if self.is_hard(name):
                return "0"
            return None

        eb = ExprBuilder(self.values, self.producers, lambda n: None, resolve)
        try:
            eb.value(node.inputs[0], row_idx + ("col",))
        except CodegenError:
            return False
        del R
        return ok

    @staticmethod
    def _row_index(src_sizes) -> tuple[str, ...]:
        lead = src_sizes[:-1]
        return tuple(delinearise("row", lead)) if lead else ()

    def _reduced_row_index(self, name: str, row_idx: tuple[str, ...]) -> tuple[str, ...]:
        node = self.producers[name]
        keep = bool(node.attrs.get("keepdims", False))
        return row_idx + ("0",) if keep else row_idx

    # ------------------------------------------------------------------ requests and owners

    def _build_steps(self) -> list[Step]:
        # 1. requests: soft graph outputs and soft GEMM operand bases
        requests: list[str] = []
        gemm_ops: dict[str, tuple] = {}
        for kind, obj in self.raw:
            if kind != "gemm":
                continue
            node = obj
            dt = node.output.dtype.name
            if dt not in ("float32", "int32"):
                raise CodegenError(f"matmul in {dt} has no tensor-core lowering on B200")
            if len(self.sizes(node.inputs[0])) != 2 or len(self.sizes(node.inputs[1])) != 2:
                raise CodegenError("batched matmul is not lowered by the B200 backend")
            want_int8 = dt == "int32"
            a = self.gemm_operand(node.inputs[0], want_int8)
            b = self.gemm_operand(node.inputs[1], want_int8)
            if want_int8 and not (a[2] and b[2]):
                raise CodegenError("an int32 matmul lowers only when both operands are int8 values cast to int32")
            if not want_int8 and (self.values[a[0]].dtype.name != "float32" or self.values[b[0]].dtype.name != "float32"):
                raise CodegenError("a float32 matmul needs float32 operands")
            gemm_ops[node.name] = (a, b)
            for base, _, _ in (a, b):
                if self.is_hard(base):
                    if base not in self.inputs:
                        self.materialised.add(base)
                elif base not in requests:
                    requests.append(base)
        for o in self.outputs:
            if self.is_hard(o):
                if o not in self.inputs:
                    self.materialised.add(o)
            elif o not in requests:
                requests.append(o)
        self.gemm_ops = gemm_ops

        # 2. owners
        step_of: dict[str, int] = {}
        for k, (kind, obj) in enumerate(self.raw):
            if kind == "row":
                for m in obj.members:
                    step_of[m] = k
            else:
                step_of[obj.name] = k
        owned: dict[int, list[str]] = {}
        maps: dict[int, list[str]] = {}
        for r in requests:
            deps = self.hard_deps(r)
            latest = max((step_of.get(d, -1) for d in deps), default=-1)
            owner = None
            if latest >= 0:
                kind, obj = self.raw[latest]
                rs = self.sizes(r)
                if kind == "gemm" and rs == self.sizes(obj.name) and self._epilogue_ok(obj.name, r):
                    owner = latest
                elif kind == "row" and (rs == obj.src_sizes or rs in self._row_shapes(obj.src_sizes)):
                    if self._final_phase_ok(obj, r):
                        owner = latest
                elif kind == "red" and self._col_epilogue_ok(obj, r, deps):
                    owner = latest
            if owner is None:
                maps.setdefault(latest, []).append(r)
            else:
                owned.setdefault(owner, []).append(r)

        # 3. emission order: map steps right after the step they depend on. A request
        #    written by an earlier step is read from memory by later steps (never recomputed),
        #    so everything below walks expressions only down to that frontier.
        seq: list[tuple] = [("map", [r]) for r in maps.get(-1, [])]
        for k, (kind, obj) in enumerate(self.raw):
            seq.append((kind, obj, owned.get(k, [])))
            seq.extend(("map", [r]) for r in maps.get(k, []))
        self.request_pos = {}
        for pos, item in enumerate(seq):
            for r in (item[1] if item[0] == "map" else item[2]):
                self.request_pos[r] = pos
        self._frontier_memo = {}

        # 4. which hard values are read by a kernel other than their producer
        def note_reads(roots: list[str], own: set[str], pos: int):
            for n in roots:
                for d in self.frontier(n, pos):
                    if d not in own and d not in self.inputs and self.is_hard(d):
                        self.materialised.add(d)

        for pos, item in enumerate(seq):
            kind = item[0]
            if kind == "map":
                note_reads(item[1], set(), pos)
            elif kind == "gemm":
                note_reads(item[2], {item[1].name}, pos)
            elif kind == "row":
                members = set(item[1].members)
                note_reads([self.producers[m].inputs[0] for m in item[1].members], members, pos)
                note_reads(item[2], members, pos)
            else:
                note_reads([item[1].inputs[0]], set(), pos)

        # 5. generate the steps in order
        steps: list[Step] = []
        for pos, item in enumerate(seq):
            self._gen_pos = pos
            self._step_reads = set()
            kind = item[0]
            if kind == "map":
                new = [self._map_step(item[1])]
            elif kind == "gemm":
                new = [self._gemm_step(item[1], item[2])]
            elif kind == "row":
                new = [self._row_step(item[1], item[2])]
            else:
                new = self._reduction_steps(item[1], item[2])
            for st in new:
                st.reads = sorted(set(st.reads) | self._step_reads)
            steps.extend(new)
        if CHAIN_GEMM:
            steps = self._fuse_chains(steps)
        self.steps = steps
        return steps

    # ------------------------------------------------------------------ gemm chains

    def _chainable(self, first: Step, second: Step) -> bool:
        """Whether ``second`` may share ``first``'s launch as the second GEMM of a chain."""
        g1, g2 = first.pair_gemm, second.pair_gemm
        if g1 is None or g2 is None or g1.is_int != g2.is_int or g1.M != g2.M:
            return False
        a2 = g2.opa
        # the second GEMM's A is the first one's stored output, read whole and K-major
        if a2.value not in first.writes or a2.mn_major or (a2.rows, a2.cols) != (g1.M, g1.N):
            return False
        # nothing else of the second GEMM (B, epilogue side inputs) may come from the first
        if g2.opb.value in first.writes or (set(second.reads) - {a2.value}) & set(first.writes):
            return False
        tiles = (g1.M // 256) * (g1.N // 256) + (g2.M // 256) * (g2.N // 256)
        return tiles <= CHAIN_MAX_ITEMS

    def _prologue_ok(self, row: Step, first: Step, second: Step) -> bool:
        """Whether ``row`` can run as the row prologue of the chain (first, second): it writes
        the first GEMM's A operand whole, one warp per row, and nothing of what it writes is
        read by the chain other than through that operand's TMA loads."""
        body, a1 = row.row_body, first.pair_gemm.opa
        if body is None or len(row.launches) != 1 or a1.value not in row.writes or a1.mn_major:
            return False
        if (a1.rows, a1.cols) != (body.rows, body.cols) or body.rows % 256:
            return False
        if -(-(body.rows // 16) // NUM_SMS) > ROW_PROLOGUE_MAX_ROUNDS:
            return False
        epis = first.pair_gemm.epi_source + second.pair_gemm.epi_source
        for w in row.writes:
            if PTR(w) in epis or w in (first.pair_gemm.opb.value, second.pair_gemm.opb.value):
                return False
        return all(w == a1.value or w not in second.reads for w in row.writes)

    def _fuse_chains(self, steps: list[Step]) -> list[Step]:
        out: list[Step] = []
        i = 0
        while i < len(steps):
            if i + 1 < len(steps) and self._chainable(steps[i], steps[i + 1]):
                row = None
                if ROW_PROLOGUE and out and self._prologue_ok(out[-1], steps[i], steps[i + 1]):
                    row = out.pop()
                out.append(self._chain_step(steps[i], steps[i + 1], row))
                i += 2
            else:
                out.append(steps[i])
                i += 1
        return out

    def _chain_step(self, first: Step, second: Step, row: Step | None = None) -> Step:
        from tgcb import chain

        g1, g2 = first.pair_gemm, second.pair_gemm
        pairs = NUM_SMS // 2
        kb_elems = 128 if g1.is_int else 32  # K values per 128-byte k-block
        rows = g1.M // 256
        tn1, tn2 = g1.N // 256, g2.N // 256
        lists, _ = chain.schedule(rows * tn1, tn1, -(-g1.K // kb_elems), rows * tn2, tn2, -(-g2.K // kb_elems), pairs)
        kname = self._kname("chain")
        counters = f"{kname}_rows_done"
        # one counter per 256-row block for the second GEMM's waits, and with a row prologue as
        # many for the first GEMM's
        counter_bytes = rows * 4 * (2 if row is not None else 1)
        self.scratch[counters] = counter_bytes
        items = [t for lst in lists for t in lst]
        offs = [0]
        for lst in lists:
            offs.append(offs[-1] + len(lst))

        def table(name: str, vals: list[int]) -> str:
            body = ", ".join(str(v) for v in vals)
            return f"static __constant__ unsigned short {name}[{len(vals)}] = {{{body}}};\n"

        sched = f"Sched_{kname}"
        b = "true" if g1.is_int else "false"

        def gemm_t(g: PairGemmInfo) -> str:
            return (f"tgcb_gemm::PairGemm<{g.M}, {g.N}, {g.K}, {'true' if g.opa.mn_major else 'false'}, "
                    f"{'true' if g.opb.mn_major else 'false'}, {g.epi_name}>")

        pro = ""
        pro_t = ""
        if row is not None:
            body = row.row_body
            pro_t = f", Rows_{kname}"
            pro = (
                f"struct Rows_{kname} {{\n"
                f"  static constexpr int GROUPS = {body.rows // 16};  // groups of tgcb_gemm::EPI_WARPS rows\n"
                "  static __device__ __forceinline__ void row(const TgcbArgs& args, const long long row, const int tid) {\n"
                f"    double red_smem[{body.nred}][1][1];  // one warp per row: never written\n"
                "    const int grp = 0;\n"
                "    const bool live = true;\n"
                f"{body.lines}\n"
                "  }\n};\n"
            )
        source = (
            g1.epi_source + g2.epi_source + pro
            + table(f"{kname}_items", items) + table(f"{kname}_first", offs)
            + f"struct {sched} {{\n"
            f"  static constexpr int PAIRS = {pairs};\n"
            f"  static __device__ __forceinline__ int count(int pair, int) {{ return {kname}_first[pair + 1] - {kname}_first[pair]; }}\n"
            f"  static __device__ __forceinline__ int item(int pair, int, int i) {{ return {kname}_items[{kname}_first[pair] + i]; }}\n"
            "};\n"
            f'extern "C" __global__ void __launch_bounds__({CHAIN_THREADS}, 1) {kname}(const TgcbArgs args, '
            "const __grid_constant__ TgcbTmaDesc ta, const __grid_constant__ TgcbTmaDesc tb, "
            "const __grid_constant__ TgcbTmaDesc ta2, const __grid_constant__ TgcbTmaDesc tb2) {\n"
            f"  tgcb_gemm::gemm_chain_pair<{b}, {gemm_t(g1)}, {gemm_t(g2)}, {sched}{pro_t}>(args, &ta, &tb, &ta2, &tb2, "
            f"reinterpret_cast<unsigned*>({PTR(counters)}));\n}}\n"
        )
        launch = Launch(kname, (2 * pairs, 1, 1), (CHAIN_THREADS, 1, 1), smem=-1, gemm=(g1.opa, g1.opb), pair=True,
                        gemm2=(g2.opa, g2.opb), counters=counters, counter_bytes=counter_bytes)
        how = (f"{first.bracketing} | then {second.bracketing} | both GEMMs in one launch: {len(items)} tiles on "
               f"{pairs} SM pairs in a fixed per-pair order, a tile of the second GEMM after its 256-row block of the first")
        reads = set(first.reads) | set(second.reads)
        unused = set(g1.split_scratch) | set(g2.split_scratch)
        writes = [w for w in first.writes if w not in unused]
        writes += [w for w in second.writes if w not in first.writes and w not in unused] + [counters]
        nodes = list(first.nodes) + list(second.nodes)
        if row is not None:
            how = (f"{row.bracketing}, the rows computed inside the launch by the epilogue warps (one warp per row) "
                   f"before their first tile, a tile of the first GEMM after its 256 rows | " + how)
            reads |= set(row.reads)
            writes = list(row.writes) + [w for w in writes if w not in row.writes]
            nodes = list(row.nodes) + nodes
        return Step(
            "gemm",
            f"{first.label}+{second.label}",
            reads=sorted(reads),
            writes=writes,
            source=source,
            launches=[launch],
            bracketing=how,
            nodes=nodes,
        )

    def _row_shapes(self, src_sizes) -> list[tuple[int, ...]]:
        lead = tuple(src_sizes[:-1])
        return [lead, lead + (1,)]

    def _epilogue_ok(self, gemm: str, request: str) -> bool:
        ok = True
        ident = ("row", "col")

        def resolve(name, idx):
            nonlocal ok
            if name == gemm:
                if tuple(idx) != ident:
                    ok = False
                return "acc"
            if self.is_hard(name):
                return "0"
            return None

        eb = ExprBuilder(self.values, self.producers, lambda n: None, resolve)
        try:
            eb.value(request, ident)
        except CodegenError:
            return False
        return ok

    def _final_phase_ok(self, group: RowGroup, request: str) -> bool:
        members = set(group.members)
        row_idx = self._row_index(group.src_sizes)
        rs = self.sizes(request)
        full = rs == tuple(group.src_sizes)
        idx = row_idx + ("col",) if full else (row_idx + ("0",) if rs == tuple(group.src_sizes[:-1]) + (1,) else row_idx)
        ok = True

        def resolve(name, i):
            nonlocal ok
            if name in members:
                if tuple(i) != self._reduced_row_index(name, row_idx):
                    ok = False
                return "0"
            if self.is_hard(name):
                if not full:
                    # a row-shaped output may only read per-row values
                    ok = False
                return "0"
            return None

        eb = ExprBuilder(self.values, self.producers, lambda n: None, resolve)
        try:
            eb.value(request, idx)
        except CodegenError:
            return False
        return ok

    # ------------------------------------------------------------------ kernel sources

    def _kname(self, stem: str) -> str:
        self.kernel_count += 1
        return f"tgcb_{stem}_{self.kernel_count}"

    def _pointer_of(self, name: str) -> str | None:
        """Base pointer of ``name`` if the kernel being generated reads it from memory."""
        if name in self.inputs or name in self.materialised or self.request_pos.get(name, 1 << 30) < self._gen_pos:
            self._step_reads.add(name)
            return PTR(name)
        return None

    def frontier(self, name: str, pos: int) -> frozenset[str]:
        """Memory-resident values an expression for ``name`` reads when generated at step ``pos``:
        hard values, and requests materialised by an earlier step."""
        key = (name, pos)
        if key in self._frontier_memo:
            return self._frontier_memo[key]
        if self.is_hard(name) or self.request_pos.get(name, 1 << 30) < pos:
            out = frozenset([name])
        else:
            acc: set[str] = set()
            for i in self.producers[name].inputs:
                acc |= self.frontier(i, pos)
            out = frozenset(acc)
        self._frontier_memo[key] = out
        return out

    def _map_step(self, names: list[str]) -> Step:
        out_sizes = self.sizes(names[0])
        total = max(1, _prod(out_sizes))
        kname = self._kname("map")
        body: list[str] = []
        reads: set[str] = set()
        T = 256
        unroll = 4
        for u in range(unroll):
            e = f"(base + {u}LL * stride)"
            idx = tuple(delinearise(e, out_sizes)) if out_sizes else ()
            eb = ExprBuilder(self.values, self.producers, self._pointer_of, indent="      ")
            stores = []
            for n in names:
                v = eb.value(n, idx)
                stores.append(f"      reinterpret_cast<{ctype(self.values[n].dtype)}*>({PTR(n)})[{e}] = {v};")
            reads |= eb.loads
            body.append(f"    if ({e} < {total}LL) {{")
            body.extend(eb.lines)
            body.extend(stores)
            body.append("    }")
        blocks = max(1, min((total + T * unroll - 1) // (T * unroll), NUM_SMS * 16))
        src = (
            f'extern "C" __global__ void __launch_bounds__({T}) {kname}(const TgcbArgs args) {{\n'
            f"  const long long stride = (long long)gridDim.x * blockDim.x;\n"
            f"  for (long long base = (long long)blockIdx.x * blockDim.x + threadIdx.x; base < {total}LL;"
            f" base += {unroll}LL * stride) {{\n" + "\n".join(body) + "\n  }\n}\n"
        )
        return Step(
            "map",
            ",".join(names),
            reads=sorted(reads),
            writes=list(names),
            source=src,
            launches=[Launch(kname, (blocks, 1, 1), (T, 1, 1))],
            nodes=list(names),
        )

    def _row_step(self, group: RowGroup, requests: list[str]) -> Step:
        ss = tuple(group.src_sizes)
        C = ss[-1]
        R = _prod(ss[:-1])
        T = row_threads(C, R)
        W = T // 32
        npt = (C + T - 1) // T
        unrolled = npt <= 32
        members = group.members
        members_set = set(members)
        max_phase = max(group.phase.values())
        row_idx = self._row_index(ss)
        kname = self._kname("row")
        full_req = [r for r in requests if self.sizes(r) == ss]
        row_req = [r for r in requests if self.sizes(r) != ss]
        reads: set[str] = set()
        lines: list[str] = []
        hoisted: list[str] = []  # the standalone kernel's lines, first-phase loads moved up
        nred = len(members)
        slot = {m: k for k, m in enumerate(members)}

        def member_resolve(name, idx):
            if name in members_set:
                return f"red_{slot[name]}"
            return None

        shared_eb = ExprBuilder(self.values, self.producers, self._pointer_of, member_resolve, indent="    ")
        RPB = ROW_BLOCK // T  # rows side by side in one CTA, T threads each

        def col_expr(k):
            return f"((long long)tid + {k * T}LL)" if unrolled else "col"

        for phase in range(1, max_phase + 1):
            pm = [m for m in members if group.phase[m] == phase]
            accs = {}
            for m in pm:
                node = self.producers[m]
                t = ctype(node.output.dtype)
                if node.op.name == "max":
                    init = "-INFINITY" if t in ("float", "double") else ("(-2147483647-1)" if t == "int" else "(-9223372036854775807LL-1)")
                else:
                    init = f"({t})0"
                accs[m] = (f"acc_{slot[m]}", t, node.op.name)
                lines.append(f"    {t} acc_{slot[m]} = {init};")
            if unrolled:
                eb = shared_eb
                ks = range(npt)
            else:
                eb = ExprBuilder(self.values, self.producers, self._pointer_of, member_resolve, indent="      ")
                ks = [0]
                lines.append(f"    for (long long col = tid; col < {C}LL; col += {T}LL) {{")
            phase_start = len(lines)
            for k in ks:
                col = col_expr(k)
                colc = f"tgcb_min_ll({col}, {C - 1}LL)" if (unrolled and C % T) else col
                for m in pm:
                    node = self.producers[m]
                    v = eb.value(node.inputs[0], row_idx + (colc,))
                    acc, t, opn = accs[m]
                    if opn == "max":
                        upd = f"(({acc}) != ({acc}) || ({acc}) > ({v})) ? ({acc}) : ({t})({v})"
                    else:
                        upd = f"{acc} + ({t})({v})"
                    guard = f"({col} < {C}LL) ? ({upd}) : {acc}" if (unrolled and C % T) else upd
                    eb.emit(f"{acc} = {guard};")
                if unrolled:
                    lines.extend(eb.lines)
                    eb.lines = []
            if unrolled and phase == 1:
                # load offsets are index arithmetic on tid, row and constants only, so every
                # load of the phase can move ahead of the phase's arithmetic
                body = lines[phase_start:]
                hoisted = lines[:phase_start] + [ln for ln in body if _LOAD_LINE.match(ln)] + [
                    ln for ln in body if not _LOAD_LINE.match(ln)
                ]
            if not unrolled:
                lines.extend(eb.lines)
                lines.append("    }")
            # combine the row's partials with the declared tree bracketing
            for m in pm:
                acc, t, opn = accs[m]
                fn = "tgcb_group_max" if opn == "max" else "tgcb_group_sum"
                lines.append(f"    {t} red_{slot[m]} = {fn}<{t}, {W}>({acc}, reinterpret_cast<{t}*>(red_smem[{slot[m]}][grp]), tid);")
                if opn == "mean":
                    lines.append(f"    red_{slot[m]} = red_{slot[m]} / ({t}){C};")
        # final phase: full-shaped requests
        if full_req:
            if unrolled:
                eb = shared_eb
                for k in range(npt):
                    col = col_expr(k)
                    colc = f"tgcb_min_ll({col}, {C - 1}LL)" if C % T else col
                    for r in full_req:
                        v = eb.value(r, row_idx + (colc,))
                        st = f"reinterpret_cast<{ctype(self.values[r].dtype)}*>({PTR(r)})[row * {C}LL + {col}] = {v};"
                        eb.emit(f"if (live && {col} < {C}LL) {st}" if C % T else f"if (live) {st}")
                    lines.extend(eb.lines)
                    eb.lines = []
            else:
                eb = ExprBuilder(self.values, self.producers, self._pointer_of, member_resolve, indent="      ")
                lines.append(f"    for (long long col = tid; col < {C}LL; col += {T}LL) {{")
                for r in full_req:
                    v = eb.value(r, row_idx + ("col",))
                    eb.emit(f"if (live) reinterpret_cast<{ctype(self.values[r].dtype)}*>({PTR(r)})[row * {C}LL + col] = {v};")
                lines.extend(eb.lines)
                lines.append("    }")
        # per-row results: materialised reductions and row-shaped requests
        row_stores = [m for m in members if m in self.materialised] + row_req
        if row_stores:
            eb = ExprBuilder(self.values, self.producers, self._pointer_of, member_resolve, indent="      ")
            lines.append("    if (tid == 0 && live) {")
            for r in row_stores:
                rs = self.sizes(r)
                idx = row_idx + ("0",) if len(rs) == len(ss) else row_idx
                v = eb.value(r, idx)
                eb.emit(f"reinterpret_cast<{ctype(self.values[r].dtype)}*>({PTR(r)})[row] = {v};")
            lines.extend(eb.lines)
            lines.append("    }")
        if W > 1:
            lines.append("    __syncthreads();")
        reads |= shared_eb.loads
        row_blocks = (R + RPB - 1) // RPB
        grid = max(1, min(row_blocks, NUM_SMS * (2048 // ROW_BLOCK) * 2))
        kernel_lines = hoisted + lines[len(hoisted):] if (hoisted and ROW_HOIST_LOADS) else lines
        src = (
            f'extern "C" __global__ void __launch_bounds__({ROW_BLOCK}) {kname}(const TgcbArgs args) {{\n'
            f"  __shared__ double red_smem[{nred}][{RPB}][{W}];\n"
            f"  const int tid = threadIdx.x % {T};\n"
            f"  const int grp = threadIdx.x / {T};\n"
            f"  for (long long rb = (long long)blockIdx.x * {RPB}; rb < {R}LL; rb += (long long)gridDim.x * {RPB}) {{\n"
            f"    const bool live = rb + grp < {R}LL;\n"
            f"    const long long row = live ? rb + grp : {R - 1}LL;\n"
            + "\n".join(kernel_lines)
            + "\n  }\n}\n"
        )
        writes = [m for m in members if m in self.materialised] + list(requests)
        step = Step(
            "row",
            ",".join(members),
            reads=sorted(reads),
            writes=writes,
            source=src,
            launches=[Launch(kname, (grid, 1, 1), (ROW_BLOCK, 1, 1))],
            bracketing=f"row tree: {T} threads per row, thread t sums columns t, t+{T}, ... in order; "
            f"lanes combined by xor tree (1,2,4,8,16); {W} warp partials combined as a balanced tree",
            nodes=list(members) + list(requests),
        )
        if T == 32 and unrolled:
            # one warp per row and no shared-memory partials: the same body can run inside a
            # GEMM chain launch, one row per epilogue warp (a row prologue)
            step.row_body = RowBody("\n".join(lines), nred, R, C)
        return step

    def _reduction_steps(self, node, owned: list[str] | None = None) -> list[Step]:
        kind = self.reduction_kind(node)
        if kind == "col":
            return self._col_steps(node, owned or [])
        if owned:
            raise CodegenError("only column reductions take requests")
        if kind == "full":
            return self._full_steps(node)
        return [self._naive_step(node)]

    def _acc_update(self, opn: str, acc: str, v: str, t: str) -> str:
        if opn == "max":
            return f"{acc} = (({acc}) != ({acc}) || ({acc}) > ({v})) ? ({acc}) : ({t})({v});"
        return f"{acc} = {acc} + ({t})({v});"

    def _init(self, opn: str, t: str) -> str:
        if opn == "max":
            return "-INFINITY" if t in ("float", "double") else "(-2147483647-1)"
        return f"({t})0"

    def _col_epilogue_ok(self, node, r: str, deps) -> bool:
        """Whether request ``r`` can be computed where a column reduction's final values are: it
        depends on nothing but that reduction's result, element for element (a reshape or an
        elementwise function of it, same element count)."""
        if self.reduction_kind(node) != "col" or set(deps) != {node.name}:
            return False
        if _prod(self.sizes(r)) != _prod(self.sizes(node.name)):
            return False
        try:
            self._col_request_lines(node, r, "v")
        except CodegenError:
            return False
        return True

    def _col_request_lines(self, node, r: str, fin: str) -> list[str]:
        """Statements that store request ``r`` at column c from the reduction's value ``fin``."""
        red_sizes = self.sizes(node.name)

        def resolve(name, idx):
            if name != node.name:
                return None
            if tuple(i for i, n in zip(idx, red_sizes, strict=True) if n != 1) != ("c",):
                raise CodegenError("not aligned with the reduction's columns")
            return fin

        eb = ExprBuilder(self.values, self.producers, lambda n: None, resolve, indent="  ")
        v = eb.value(r, tuple(delinearise("c", self.sizes(r))))
        t = ctype(self.values[r].dtype)
        return eb.lines + [f"  reinterpret_cast<{t}*>({PTR(r)})[c] = {v};"]

    def _col_steps(self, node, owned: list[str] | None = None) -> list[Step]:
        """Reduction over axis 0 of [R, C]: P row partitions summed sequentially, then the P
        partials in order. Requests owned by the step (element-wise functions or reshapes of the
        result, such as a bias gradient's reshape) are stored by the final kernel too."""
        name = node.name
        src = node.inputs[0]
        R, C = self.sizes(src)
        t = ctype(node.output.dtype)
        opn = node.op.name
        cblocks = (C + 255) // 256
        P, L = col_split(R, C)
        scratch = f"{name}__partials"
        self.scratch[scratch] = P * C * 8
        k1, k2 = self._kname("colpart"), self._kname("colfinal")
        UNROLL = 8
        eb = ExprBuilder(self.values, self.producers, self._pointer_of, indent="    ")
        vals = [eb.value(src, (f"(r + {u})", "c")) for u in range(UNROLL)]
        # loads of UNROLL rows are independent; the additions stay in row order
        body = "\n".join(eb.lines + ["    " + self._acc_update(opn, "acc", v, t) for v in vals])
        eb1 = ExprBuilder(self.values, self.producers, self._pointer_of, indent="    ")
        v1 = eb1.value(src, ("r", "c"))
        body1 = "\n".join(eb1.lines)
        s1 = (
            f'extern "C" __global__ void __launch_bounds__(256) {k1}(const TgcbArgs args) {{\n'
            f"  const long long c = (long long)blockIdx.x * 256 + threadIdx.x;\n"
            f"  if (c >= {C}LL) return;\n"
            f"  const long long r0 = (long long)blockIdx.y * {L}LL;\n"
            f"  const long long r1 = tgcb_min_ll(r0 + {L}LL, {R}LL);\n"
            f"  {t} acc = {self._init(opn, t)};\n"
            f"  long long r = r0;\n"
            f"  for (; r + {UNROLL} <= r1; r += {UNROLL}) {{\n{body}\n  }}\n"
            f"  for (; r < r1; ++r) {{\n{body1}\n    {self._acc_update(opn, 'acc', v1, t)}\n  }}\n"
            f"  reinterpret_cast<{t}*>({PTR(scratch)})[blockIdx.y * {C}LL + c] = acc;\n}}\n"
        )
        fin = f"acc / ({t}){R}" if opn == "mean" else "acc"
        s2 = (
            f'extern "C" __global__ void __launch_bounds__(256) {k2}(const TgcbArgs args) {{\n'
            f"  const long long c = (long long)blockIdx.x * 256 + threadIdx.x;\n"
            f"  if (c >= {C}LL) return;\n"
            f"  const {t}* part = reinterpret_cast<const {t}*>({PTR(scratch)});\n"
            f"  {t} acc = {self._init(opn, t)};\n"
            f"  for (int p = 0; p < {P}; ++p) {{ const {t} v = part[p * {C}LL + c]; {self._acc_update(opn, 'acc', 'v', t)} }}\n"
            f"  const {t} fin = {fin};\n"
            f"  reinterpret_cast<{t}*>({PTR(name)})[c] = fin;\n"
            + "".join(line + "\n" for r in owned for line in self._col_request_lines(node, r, "fin"))
            + "}\n"
        )
        reads: list[str] = []  # recorded by _pointer_of while generating
        self.materialised.add(name)
        return [
            Step(
                "colreduce",
                name,
                reads=reads,
                writes=[scratch, name] + list(owned),
                source=s1 + "\n" + s2,
                launches=[
                    Launch(k1, (cblocks, P, 1), (256, 1, 1)),
                    Launch(k2, (cblocks, 1, 1), (256, 1, 1)),
                ],
                bracketing=f"partitioned: {P} row blocks of {L} summed sequentially, then the {P} partials in order",
                nodes=[name] + list(owned),
            )
        ]

    def _full_steps(self, node) -> list[Step]:
        """Reduction over every axis: G contiguous chunks, each a block tree, then a tree over G."""
        name = node.name
        src = node.inputs[0]
        ss = self.sizes(src)
        n = max(1, _prod(ss))
        t = ctype(node.output.dtype)
        opn = node.op.name
        T = 256
        G = max(1, min(NUM_SMS * 4, (n + T * 8 - 1) // (T * 8)))
        chunk = (n + G - 1) // G
        G = (n + chunk - 1) // chunk
        scratch = f"{name}__partials"
        self.scratch[scratch] = G * 8
        k1, k2 = self._kname("fullpart"), self._kname("fullfinal")
        eb = ExprBuilder(self.values, self.producers, self._pointer_of, indent="    ")
        v = eb.value(src, tuple(delinearise("e", ss)) if ss else ())
        body = "\n".join(eb.lines)
        fn = "tgcb_block_max" if opn == "max" else "tgcb_block_sum"
        s1 = (
            f'extern "C" __global__ void __launch_bounds__({T}) {k1}(const TgcbArgs args) {{\n'
            f"  __shared__ double red_smem[{T // 32}];\n"
            f"  const long long e0 = (long long)blockIdx.x * {chunk}LL;\n"
            f"  const long long e1 = min(e0 + {chunk}LL, {n}LL);\n"
            f"  {t} acc = {self._init(opn, t)};\n"
            f"  for (long long e = e0 + threadIdx.x; e < e1; e += {T}LL) {{\n{body}\n    {self._acc_update(opn, 'acc', v, t)}\n  }}\n"
            f"  acc = {fn}<{t}, {T // 32}>(acc, reinterpret_cast<{t}*>(red_smem));\n"
            f"  if (threadIdx.x == 0) reinterpret_cast<{t}*>({PTR(scratch)})[blockIdx.x] = acc;\n}}\n"
        )
        fin = f"acc / ({t}){n}" if opn == "mean" else "acc"
        s2 = (
            f'extern "C" __global__ void __launch_bounds__({T}) {k2}(const TgcbArgs args) {{\n'
            f"  __shared__ double red_smem[{T // 32}];\n"
            f"  const {t}* part = reinterpret_cast<const {t}*>({PTR(scratch)});\n"
            f"  {t} acc = {self._init(opn, t)};\n"
            f"  for (int g = threadIdx.x; g < {G}; g += {T}) {{ const {t} v = part[g]; {self._acc_update(opn, 'acc', 'v', t)} }}\n"
            f"  acc = {fn}<{t}, {T // 32}>(acc, reinterpret_cast<{t}*>(red_smem));\n"
            f"  if (threadIdx.x == 0) reinterpret_cast<{t}*>({PTR(name)})[0] = {fin};\n}}\n"
        )
        reads: list[str] = []  # recorded by _pointer_of while generating
        self.materialised.add(name)
        return [
            Step(
                "fullreduce",
                name,
                reads=reads,
                writes=[scratch, name],
                source=s1 + "\n" + s2,
                launches=[Launch(k1, (G, 1, 1), (T, 1, 1)), Launch(k2, (1, 1, 1), (T, 1, 1))],
                bracketing=f"{G} chunks of {chunk}: thread-strided sequential sums, block tree per chunk, "
                f"then thread-strided sums of the partials and one block tree",
                nodes=[name],
            )
        ]

    def _naive_step(self, node) -> Step:
        """Any other axis set: one thread per output element, sequential over the reduced indices."""
        name = node.name
        src = node.inputs[0]
        ss = self.sizes(src)
        axes = ir.normalise_axes(node.attrs["axes"], len(ss))
        keep = bool(node.attrs.get("keepdims", False))
        kept_axes = [a for a in range(len(ss)) if a not in axes]
        out_n = max(1, _prod([ss[a] for a in kept_axes]))
        red_sizes = [ss[a] for a in axes]
        red_n = max(1, _prod(red_sizes))
        t = ctype(node.output.dtype)
        opn = node.op.name
        kname = self._kname("reduce")
        out_idx = delinearise("o", [ss[a] for a in kept_axes]) if kept_axes else ()
        red_idx = delinearise("q", red_sizes) if red_sizes else ()
        full_idx = [""] * len(ss)
        for a, e in zip(kept_axes, out_idx, strict=True):
            full_idx[a] = e
        for a, e in zip(axes, red_idx, strict=True):
            full_idx[a] = e
        eb = ExprBuilder(self.values, self.producers, self._pointer_of, indent="    ")
        v = eb.value(src, tuple(full_idx))
        fin = f"acc / ({t}){red_n}" if opn == "mean" else "acc"
        src_code = (
            f'extern "C" __global__ void __launch_bounds__(256) {kname}(const TgcbArgs args) {{\n'
            f"  const long long o = (long long)blockIdx.x * 256 + threadIdx.x;\n"
            f"  if (o >= {out_n}LL) return;\n"
            f"  {t} acc = {self._init(opn, t)};\n"
            f"  for (long long q = 0; q < {red_n}LL; ++q) {{\n" + "\n".join(eb.lines)
            + f"\n    {self._acc_update(opn, 'acc', v, t)}\n  }}\n"
            f"  reinterpret_cast<{t}*>({PTR(name)})[o] = {fin};\n}}\n"
        )
        del keep
        self.materialised.add(name)
        return Step(
            "reduce",
            name,
            reads=[],
            writes=[name],
            source=src_code,
            launches=[Launch(kname, ((out_n + 255) // 256, 1, 1), (256, 1, 1))],
            bracketing="sequential over the reduced indices in row-major order",
            nodes=[name],
        )

    # ------------------------------------------------------------------ gemm

    def _gemm_step(self, node, requests: list[str]) -> Step:
        name = node.name
        (a_base, a_flip, _), (b_base, b_flip, _) = self.gemm_ops[name]
        M, K = self.sizes(node.inputs[0])
        _, N = self.sizes(node.inputs[1])
        is_int = node.output.dtype.name == "int32"
        eb_bytes = 1 if is_int else 4
        a_rows, a_cols = self.sizes(a_base)
        b_rows, b_cols = self.sizes(b_base)
        # A is [M, K]: row-major base [M, K] is K-major; a flipped base [K, M] is M-major.
        opa = GemmOperand(a_base, a_rows, a_cols, a_flip, eb_bytes)
        # B is [K, N]: row-major base [K, N] is N-major; a flipped base [N, K] is K-major.
        opb = GemmOperand(b_base, b_rows, b_cols, not b_flip, eb_bytes)
        stores = list(requests)
        if name in self.materialised:
            stores.insert(0, name)
        kname = self._kname("gemm")
        acc_t = "int" if is_int else "float"

        # The epilogue runs once per output element (row, col) with the accumulator value;
        # the kernel calls it with consecutive lanes on consecutive columns, so every load of
        # a side input and every store below is coalesced along the row.
        def resolve(n, idx):
            if n == name:
                return "acc"
            return None

        # A TF32 GEMM's epilogue is compared at TF32 tolerance, so it may use the approximate
        # exp/tanh/sigmoid and fused multiply-adds; the int8 epilogue stays exact.
        eb = ExprBuilder(self.values, self.producers, self._pointer_of, resolve, indent="    ", approx=not is_int)
        st = []
        for r in stores:
            v = eb.value(r, ("row", "col"))
            st.append(f"    reinterpret_cast<{ctype(self.values[r].dtype)}*>({PTR(r)})[row * {N}LL + col] = {v};")
        # Side-input loads never depend on the accumulator: they go into load(), which the
        # kernel issues ahead of time (before waiting for the tile, and one chunk ahead while
        # the previous chunk computes); apply() does the arithmetic and the stores.
        loads, comps = [], []
        for line in eb.lines:
            m = _LOAD_LINE.match(line)
            # only full-matrix side inputs are worth registers ahead of time; row/column
            # vectors (biases, scales) are L1 hits and stay inline
            if m and "row" in m.group(3) and "col" in m.group(3):
                loads.append(m.groups())
            else:
                comps.append(line)
        if not is_int:
            comps = contract_fma(comps, st)
        members = "".join(f"    {t} {n};\n" for t, n, _ in loads) or "    int unused;\n"
        load_body = "".join(f"      L.{n} = {e};\n" for t, n, e in loads)
        fetched = {n for _, n, _ in loads}
        comp_body = "\n".join(
            _LOAD_NAME.sub(lambda m: f"L.{m.group(1)}" if m.group(1) in fetched else m.group(1), ln) for ln in comps + st
        )
        epi_name = f"Epi_{kname}"
        # every 128 x 256 tile lies inside the output: the epilogue needs no bounds checks
        whole_tiles = M % 128 == 0 and N % 256 == 0
        vec4 = self._gemm_vec4_epilogue(name, stores, M, N, acc_t, whole_tiles)
        epi = (
            f"struct {epi_name} {{\n"
            + (vec4 or "  static constexpr bool VEC4 = false;\n")
            + f"  struct Loads {{\n{members}  }};\n"
            f"  static __device__ __forceinline__ Loads load(const TgcbArgs& args, long long row, long long col) {{\n"
            f"    Loads L;\n"
            + (f"    {{\n{load_body}    }}\n" if whole_tiles else f"    if (row < {M}LL && col < {N}LL) {{\n{load_body}    }}\n")
            + f"    return L;\n  }}\n"
            f"  static __device__ __forceinline__ void apply(const TgcbArgs& args, long long row, long long col, const {acc_t} acc, const Loads& L) {{\n"
            + ("" if whole_tiles else f"    if (row >= {M}LL || col >= {N}LL) return;\n") + comp_body + "\n  }\n};\n"
        )
        reads = {a_base, b_base}  # plus whatever the epilogue loads (recorded by _pointer_of)
        tma_ok = all((op.cols * op.elem_bytes) % 16 == 0 for op in (opa, opb))
        split_scratch: tuple[str, ...] = ()  # a K split's workspace and counters
        if tma_ok:
            # Whole 256 x 256 tiles with the four-column epilogue run on SM pairs (two CTAs of a
            # cluster share one tcgen05.mma.cta_group::2 tile); everything else on single SMs.
            pair = vec4 is not None and M % 256 == 0 and N % 256 == 0 and PAIR_GEMM
            split = self._k_split(M, N, K, is_int) if pair else 1
            body = "gemm_body_pair" if pair else "gemm_body"
            targs = (f"{M}, {N}, {K}, {'true' if is_int else 'false'}, {'true' if opa.mn_major else 'false'}, "
                     f"{'true' if opb.mn_major else 'false'}, {epi_name}")
            head = (f'extern "C" __global__ void __launch_bounds__({GEMM_THREADS}, 1) {kname}(const TgcbArgs args, '
                    "const __grid_constant__ TgcbTmaDesc ta, const __grid_constant__ TgcbTmaDesc tb) {\n")
            counters, counter_bytes = None, 0
            if split > 1:
                # K in `split` slices: partials in an arena workspace, one counter per 32 x 64
                # region of every output tile (zeroed by the runtime before each launch)
                ws, counters = f"{kname}_partials", f"{kname}_regions"
                counter_bytes = (M // 256) * (N // 256) * 32 * 4
                self.scratch[ws] = split * M * N * 4
                self.scratch[counters] = counter_bytes
                split_scratch = (ws, counters)
                stores = stores + list(split_scratch)
                kernel = head + (f"  tgcb_gemm::gemm_split_pair<{targs}, {split}>(args, &ta, &tb, (void*)({PTR(ws)}), "
                                 f"reinterpret_cast<unsigned*>({PTR(counters)}));\n}}\n")
            else:
                kernel = head + f"  tgcb_gemm::{body}<{targs}>(args, &ta, &tb);\n}}\n"
            if pair:
                grid = 2 * max(1, min((M // 256) * (N // 256) * split, NUM_SMS // 2))
            else:
                grid = max(1, min(((M + 127) // 128) * ((N + 255) // 256), NUM_SMS))
            launch = Launch(kname, (grid, 1, 1), (GEMM_THREADS, 1, 1), smem=-1, gemm=(opa, opb), pair=pair,
                            counters=counters, counter_bytes=counter_bytes)
            how = "tcgen05." + ("kind::i8, int32 accumulator in TMEM (exact)" if is_int else "kind::tf32, fp32 accumulator in TMEM, K in steps of 8")
            if pair:
                how += "; SM pairs (cta_group::2), 256 x 256 tiles"
            if split > 1:
                how += (f"; K cut into {split} equal slices, each slice's partial stored, the slices of every "
                        f"32 x 64 region summed in slice order by whichever slice finishes last")
        else:
            pair = False
            kernel = self._gemm_simt_kernel(kname, epi_name, M, N, K, is_int, a_base, a_flip, b_base, b_flip)
            launch = Launch(kname, ((M * ((N + 15) // 16) + 127) // 128, 1, 1), (128, 1, 1))
            how = "SIMT fallback for rows TMA cannot tile: sequential over K with tf32-truncated operands"
        return Step(
            "gemm",
            name,
            reads=sorted(reads),
            writes=stores,
            source=epi + kernel,
            launches=[launch],
            bracketing=how,
            nodes=[name] + list(requests),
            # a chain, when this GEMM joins one, runs it unsplit (its tiles fill the other GEMM's waves)
            pair_gemm=PairGemmInfo(M, N, K, is_int, opa, opb, epi_name, epi, split_scratch) if pair else None,
        )

    def _k_split(self, M: int, N: int, K: int, is_int: bool) -> int:
        """K slices for an SM-pair GEMM with at most half as many output tiles as SM pairs: the
        most slices (up to SPLIT_MAX, at least SPLIT_MIN_KBLOCKS k-blocks each) whose items
        all run at once. All slices then run side by side, so every slice's operands are read
        from HBM once and shared through L2 by its tiles. With more items than pairs the
        slices of one tile run in different rounds and re-read their operands: the training
        step's weight gradients (64 tiles, 8 slices in 7 rounds) measured 3% slower split."""
        pairs = NUM_SMS // 2
        tiles = (M // 256) * (N // 256)
        if not K_SPLIT or 2 * tiles > pairs:
            return 1
        kb = -(-K // (128 if is_int else 32))
        best = 1
        for s in range(2, SPLIT_MAX + 1):
            if kb % s == 0 and kb // s >= SPLIT_MIN_KBLOCKS and tiles * s <= pairs:
                best = s
        return best

    def _gemm_vec4_epilogue(self, name: str, stores: list[str], M: int, N: int, acc_t: str,
                            whole_tiles: bool = False) -> str | None:
        """Members of the epilogue struct for four consecutive columns per call (VEC4).

        The tcgen05 kernel hands ``apply4`` one row and columns col..col+3 (col a multiple of
        4): side inputs that are contiguous along the row arrive as one 16-byte load, column
        vectors (biases, scales) too, values that do not depend on the column once, and every
        store is one 16-byte store. The arithmetic is the scalar epilogue's, written out once
        per column. None when N or a stored type does not allow 16-byte accesses.
        """
        vec_t = {"float": "float4", "int": "int4"}
        if N % 4 or any(ctype(self.values[r].dtype) not in vec_t for r in stores):
            return None
        per_col = []
        for j in range(4):
            def resolve(n, idx, j=j):
                return f"acc_{j}" if n == name else None

            eb = ExprBuilder(self.values, self.producers, self._pointer_of, resolve, indent="    ", approx=acc_t == "float")
            vals = [eb.value(r, ("row", f"c{j}")) for r in stores]
            per_col.append((eb, vals))

        def rename(text: str, j: int) -> str:
            return re.sub(r"\b(ld|e|cat)_(\d+)\b", lambda m: f"{m.group(1)}_{m.group(2)}_{j}", text)

        members, body, sub = [], [], {}
        infos = [eb.load_info for eb, _ in per_col]
        for k, (var, t, ptr, off) in enumerate(infos[0]):
            offs = [infos[j][k][3] for j in range(4)]
            if all("c" + str(j) not in offs[j] for j in range(4)) and len(set(offs)) == 1:
                members.append(f"    {t} {var};")
                body.append(f"      L.{var} = __ldg(reinterpret_cast<const {t}*>({ptr}) + {off});")
                for j in range(4):
                    sub[f"{var}_{j}"] = f"L.{var}"
                continue
            m = re.fullmatch(r"\(c0(?: \+ \(row\)\*(\d+)LL)?\)", off)
            if t in vec_t and m and (m.group(1) is None or int(m.group(1)) % 4 == 0) and all(
                offs[j] == off.replace("c0", f"c{j}") for j in range(4)
            ):
                members.append(f"    {vec_t[t]} {var};")
                body.append(f"      L.{var} = __ldg(reinterpret_cast<const {vec_t[t]}*>(reinterpret_cast<const {t}*>({ptr}) + {off}));")
                for j, lane in enumerate("xyzw"):
                    sub[f"{var}_{j}"] = f"L.{var}.{lane}"
                continue
            for j in range(4):
                vj, tj, pj, oj = infos[j][k]
                members.append(f"    {tj} {vj}_{j};")
                body.append(f"      L.{vj}_{j} = __ldg(reinterpret_cast<const {tj}*>({pj}) + {oj});")
                sub[f"{vj}_{j}"] = f"L.{vj}_{j}"
        comps = []
        for j, (eb, vals) in enumerate(per_col):
            lines = [ln for ln in eb.lines if not _LOAD_LINE.match(ln)]
            if acc_t == "float":
                lines = contract_fma(lines, vals)
            comps.extend(rename(ln, j) for ln in lines)
        finals = [[rename(v, j) for v in vals] for j, (_, vals) in enumerate(per_col)]
        for i, r in enumerate(stores):
            t = ctype(self.values[r].dtype)
            parts = ", ".join(f"({t})({finals[j][i]})" for j in range(4))
            comps.append(
                f"    *reinterpret_cast<{vec_t[t]}*>(reinterpret_cast<{t}*>({PTR(r)}) + (row * {N}LL + col)) = "
                f"make_{vec_t[t]}({parts});"
            )
        pattern = re.compile(r"\b(?:ld|e|cat)_\d+_\d\b")
        comp_body = "\n".join(pattern.sub(lambda m: sub.get(m.group(0), m.group(0)), ln) for ln in comps)
        cols = "    const long long c0 = col, c1 = col + 1, c2 = col + 2, c3 = col + 3;\n"
        accs = "".join(f"    const {acc_t} acc_{j} = acc.{lane};\n" for j, lane in enumerate("xyzw"))
        member_text = "\n".join(members) + "\n" if members else "    int unused;\n"
        return (
            "  static constexpr bool VEC4 = true;\n"
            f"  struct Loads4 {{\n{member_text}  }};\n"
            "  static __device__ __forceinline__ Loads4 load4(const TgcbArgs& args, long long row, long long col) {\n"
            "    Loads4 L;\n"
            + cols
            + ("    {\n" if whole_tiles else f"    if (row < {M}LL && col < {N}LL) {{\n") + "".join(b + "\n" for b in body) + "    }\n"
            "    return L;\n  }\n"
            f"  static __device__ __forceinline__ void apply4(const TgcbArgs& args, long long row, long long col, "
            f"const {vec_t[acc_t]} acc, const Loads4& L) {{\n"
            + ("" if whole_tiles else f"    if (row >= {M}LL || col >= {N}LL) return;\n") + cols + accs + comp_body + "\n  }\n"
        )

    def _gemm_simt_kernel(self, kname, epi_name, M, N, K, is_int, a_base, a_flip, b_base, b_flip) -> str:
        """One thread per 16 output columns of a row; used when an operand row is not 16-byte aligned."""
        et = "signed char" if is_int else "float"
        at = "int" if is_int else "float"
        a_idx = "(long long)k * %dLL + row" % M if a_flip else "row * %dLL + k" % K
        b_idx = "(long long)(col0 + j) * %dLL + k" % K if b_flip else "(long long)k * %dLL + col0 + j" % N
        if is_int:
            load_a = f"(int)reinterpret_cast<const {et}*>({PTR(a_base)})[{a_idx}]"
            load_b = f"(int)reinterpret_cast<const {et}*>({PTR(b_base)})[{b_idx}]"
            fma = "acc[j] = (int)((unsigned int)acc[j] + (unsigned int)(a * b));"
        else:
            trunc = "__uint_as_float(__float_as_uint(%s) & 0xffffe000u)"
            load_a = trunc % f"reinterpret_cast<const {et}*>({PTR(a_base)})[{a_idx}]"
            load_b = trunc % f"reinterpret_cast<const {et}*>({PTR(b_base)})[{b_idx}]"
            fma = "acc[j] = fmaf(a, b, acc[j]);"
        groups = (N + 15) // 16
        return (
            f'extern "C" __global__ void __launch_bounds__(128) {kname}(const TgcbArgs args) {{\n'
            f"  const long long t = (long long)blockIdx.x * 128 + threadIdx.x;\n"
            f"  if (t >= {M}LL * {groups}LL) return;\n"
            f"  const long long row = t / {groups}LL;\n"
            f"  const long long col0 = (t % {groups}LL) * 16;\n"
            f"  {at} acc[16];\n"
            f"  for (int j = 0; j < 16; ++j) acc[j] = 0;\n"
            f"  for (int k = 0; k < {K}; ++k) {{\n"
            f"    const {at} a = {load_a};\n"
            f"    for (int j = 0; j < 16; ++j) {{\n"
            f"      if (col0 + j < {N}LL) {{ const {at} b = {load_b}; {fma} }}\n"
            f"    }}\n  }}\n"
            f"  for (int j = 0; j < 16; ++j) {epi_name}::apply(args, row, col0 + j, acc[j], {epi_name}::load(args, row, col0 + j));\n}}\n"
        )


def lower(graph, order) -> Lowering:
    low = Lowering(graph, order)
    low.partition()
    return low


def gemm_flops(steps: list[Step], lowering: Lowering) -> int:
    """2*M*N*K summed over the GEMM steps."""
    total = 0
    for s in steps:
        if s.kind == "gemm":
            node = lowering.producers[s.label]
            M, K = lowering.sizes(node.inputs[0])
            N = lowering.sizes(node.inputs[1])[1]
            total += 2 * M * N * K
    return total


_ = (math, _broadcast_index)
