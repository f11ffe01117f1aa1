"""Compiling a graph for the B200 and running it: the drop-in for tgc/runtime/executor.py.

``compile_graph`` keeps tgc's pipeline up to the memory plan (validate -> exact passes ->
depth-first order -> liveness -> largest-first plan, tgc/runtime/executor.py:91-108) and
replaces ``emit`` + ``exec`` (executor.py:110-113) with: partition into kernels
(``tgcb.codegen``), plan the arena over the kernel steps, write one CUDA translation unit,
compile it with NVRTC for sm_100a (cached on disk by content hash) and bind the launches in
the C library. ``CompiledGraph`` keeps tgc's fields and calls (``graph``, ``order``,
``plan``, ``module``, ``function``, ``input_names``, ``arena_bytes``, ``new_arena``,
``__call__``, ``as_dict``).

Semantics kept from tgc (executor.py:52-88, emit.py:165-209):
* ``__call__`` checks every input is supplied (``ConfigError`` naming the missing ones) and
  runs against a fresh arena, so results of separate calls never alias.
* ``function(arena, feeds)`` runs against a caller-owned arena that is reused across calls;
  returned outputs are views of that arena and the next call overwrites them.
* Inputs are never written. A CUDA feed of the declared dtype, shape and a 256-byte aligned
  address is read in place; anything else (host tensors, other dtypes, strided views) is
  copied into the input's planned slot first, converting like ``Tensor.copy_`` does.
There is no CPU path: compiling needs the CUDA library and running needs a CUDA device.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import re
from collections.abc import Callable
from dataclasses import dataclass, field

from tgcb import _lib, codegen, ir, memory
from tgcb.codegen import Lowering, Step
from tgcb.errors import CodegenError, ConfigError, DeviceError
from tgcb.passes import default_pipeline

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")
HEADERS = ("jit_common.cuh", "gemm_sm100.cuh", "gemm_sm100_pair.cuh")
SUPPORTED_OPS = {
    "add", "sub", "mul", "div", "maximum", "minimum", "neg", "exp", "log", "sqrt", "tanh", "relu",
    "sigmoid", "reciprocal", "abs", "step", "cast", "matmul", "sum", "mean", "max", "reshape",
    "transpose", "broadcast_to", "concat", "slice", "constant", "print", "assert_finite",
}
# tgcb_gemm::SMEM_BYTES: 4 stages of (128 + 256) rows x 128 B, barriers, the epilogue
# transpose tiles (16 warps x 32 x 8 words) and 1 KB of alignment slack.
GEMM_SMEM = 4 * (128 + 256) * 128 + 256 + 16 * 32 * 8 * 4 + 1024
GEMM_PAIR_SMEM = 6 * (128 + 128) * 128 + 256 + 16 * 32 * 8 * 4 + 1024  # tgcb_gemm::P_SMEM_BYTES
_PLACEHOLDER = re.compile(r"@P<([^>]+)>@")

TORCH_DTYPES = {}


def _torch_dtype(dtype):
    import torch

    if not TORCH_DTYPES:
        TORCH_DTYPES.update(
            {
                "bool": torch.bool, "int8": torch.int8, "int32": torch.int32, "int64": torch.int64,
                "float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
                "float64": torch.float64,
            }
        )
    return TORCH_DTYPES[dtype.name]


def unsupported_operations(graph) -> list[str]:
    """Ops the backend has no lowering for (the analogue of emit.unsupported_operations)."""
    return sorted({n.op.name for n in graph.nodes} - SUPPORTED_OPS)


def can_lower(graph) -> bool:
    return not unsupported_operations(graph) and all(n.output.shape.is_static for n in graph.nodes) and all(
        v.shape.is_static for v in graph.inputs
    )


# ----------------------------------------------------------------------------- JIT cache


def cache_dir() -> str:
    d = os.environ.get("TGCB_CACHE_DIR") or os.path.join(os.path.expanduser("~"), ".cache", "tgcb")
    os.makedirs(d, exist_ok=True)
    return d


def _header_digest() -> str:
    h = hashlib.sha256()
    for name in HEADERS:
        with open(os.path.join(CSRC, name), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def compile_source(source: str) -> bytes:
    """sm_100a cubin for ``source``, from the on-disk cache when the same text was compiled before."""
    lib = _lib.load()
    key = hashlib.sha256((source + "\0" + _header_digest() + "\0" + lib.tgcb_version().decode()).encode()).hexdigest()
    path = os.path.join(cache_dir(), key + ".cubin")
    if os.path.exists(path):
        with open(path, "rb") as f:
            return f.read()
    blob = ctypes.c_void_p()
    size = ctypes.c_size_t()
    log = ctypes.c_void_p()
    rc = lib.tgcb_compile_cubin(source.encode(), CSRC.encode(), None, 0, ctypes.byref(blob), ctypes.byref(size), ctypes.byref(log))
    text = ""
    if log.value:
        text = ctypes.string_at(log.value).decode(errors="replace")
        lib.tgcb_free(log)
    if rc != _lib.TGCB_OK:
        raise CodegenError(f"{_lib.last_error()}\n{text[:6000]}")
    data = ctypes.string_at(blob.value, size.value)
    lib.tgcb_free(blob)
    tmp = f"{path}.{os.getpid()}.tmp"
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, path)
    return data


# ----------------------------------------------------------------------------- generation


@dataclass
class GeneratedModule:
    """What codegen produced: the CUDA source and everything needed to run it (cf. EmittedModule, emit.py:59-83)."""

    source: str
    arena_bytes: int
    input_names: list[str]
    output_names: list[str]
    steps: list[Step]
    offsets: dict[str, int]
    launches: list = field(default_factory=list)

    @property
    def lines(self) -> int:
        return len(self.source.splitlines())

    @property
    def kernel_names(self) -> list[str]:
        return [ln.kernel for s in self.steps for ln in s.launches]

    def as_dict(self) -> dict:
        return {
            "lines": self.lines,
            "arena_bytes": self.arena_bytes,
            "inputs": list(self.input_names),
            "outputs": list(self.output_names),
            "kernels": self.kernel_names,
            "steps": [{"kind": s.kind, "label": s.label, "bracketing": s.bracketing} for s in self.steps],
        }


def _render(lowering: Lowering, steps: list[Step], offsets: dict[str, int]) -> str:
    index = {n: i for i, n in enumerate(lowering.inputs)}

    def sub(m: re.Match) -> str:
        name = m.group(1)
        if name in index:
            return f"(args.in[{index[name]}])"
        if name not in offsets:
            raise CodegenError(f"{name} is read by a kernel but has no arena slot")
        return f"(args.arena + {offsets[name]}LL)"

    parts = ['#include "jit_common.cuh"']
    if any(s.kind == "gemm" for s in steps):
        parts.insert(0, f"#define TGCB_CHUNKED_MN {1 if codegen.CHUNKED_MN else 0}")
        parts.append('#include "gemm_sm100.cuh"')
    if any(ln.pair for s in steps for ln in s.launches):
        parts.append('#include "gemm_sm100_pair.cuh"')
    for s in steps:
        parts.append(f"// step {s.kind}: {s.label}" + (f"\n// bracketing: {s.bracketing}" if s.bracketing else ""))
        parts.append(_PLACEHOLDER.sub(sub, s.source))
    return "\n".join(parts) + "\n"


def _operand_desc(op, lowering: Lowering, offsets: dict[str, int], tile_rows: int) -> _lib.OperandDesc:
    d = _lib.OperandDesc()
    if op.value in lowering.inputs:
        d.input_index = lowering.inputs.index(op.value)
        d.arena_offset = 0
    else:
        d.input_index = -1
        d.arena_offset = offsets[op.value]
    d.elem_bytes = op.elem_bytes
    d.rows = op.rows
    d.cols = op.cols
    d.box_cols = 128 // op.elem_bytes
    # K-major: a box is tile_rows rows of 128 bytes; MN-major: one stage of K rows.
    d.box_rows = (128 // op.elem_bytes) if op.mn_major else tile_rows
    # tcgen05 reads MN-major 32-bit operands only in the 128-byte swizzle of 32-byte units.
    d.swizzle = 1 if (op.mn_major and op.elem_bytes == 4) else 0
    # Such an operand's stage is tile_rows / 32 chunks of 32 columns (4 KB each): loaded as one
    # copy through a 3-D view when the columns come in whole chunks (the kernels' chunked_mn).
    d.chunks = tile_rows // 32 if chunked_mn(op) else 0
    return d


def chunked_mn(op) -> bool:
    """Whether the GEMM kernels load this operand through a 3-D view (tgcb_gemm::chunked_mn):
    tf32, MN-major, and its contiguous extent (the M or N of the GEMM) a multiple of 32."""
    return codegen.CHUNKED_MN and op.mn_major and op.elem_bytes == 4 and op.cols % 32 == 0


def generate(graph, *, pipeline=None, optimise: bool = True) -> tuple:
    """Everything up to (not including) loading: (optimised graph, order, plan, module, lowering).

    ``graph`` may be tgc's own Graph: it is rebuilt in tgcb's IR first (``ir.adopt``)."""
    graph = ir.adopt(graph)
    ir.validate(graph)
    if not can_lower(graph):
        raise CodegenError("this graph has operations or shapes the backend cannot lower")
    if len(graph.inputs) > _lib.MAX_INPUTS:
        raise CodegenError(f"a plan takes at most {_lib.MAX_INPUTS} inputs, this graph has {len(graph.inputs)}")
    optimised = graph
    if optimise:
        chosen = pipeline or default_pipeline()
        optimised, _ = chosen.run(graph)
    order = memory.depth_first_order(optimised)
    lowering = Lowering(optimised, order)
    steps = lowering.partition()
    sizes = {v.name: v.bytes for v in optimised.inputs}
    for s in steps:
        for w in s.writes:
            if w in lowering.scratch:
                sizes[w] = lowering.scratch[w]
            else:
                sizes[w] = lowering.values[w].bytes
    step_rw = [(s.reads, s.writes) for s in steps]
    intervals = memory.intervals_for_steps(lowering.inputs, step_rw, lowering.outputs, sizes)
    plan = memory.plan_largest_first(intervals)
    memory.validate_plan(intervals, plan)
    offsets = {a.name: a.offset for a in plan.allocations}
    source = _render(lowering, steps, offsets)
    launches = []
    for s in steps:
        for ln in s.launches:
            d = _lib.LaunchDesc()
            d.kernel = ln.kernel.encode()
            d.grid = (ctypes.c_uint32 * 3)(*ln.grid)
            d.block = (ctypes.c_uint32 * 3)(*ln.block)
            if ln.gemm is not None:
                # 1: one-SM kernel; 2: two-SM kernel, launched as clusters of two CTAs, each of
                # which stages 128 columns of B; 3: a chain of two two-SM GEMMs in one launch
                d.is_gemm = 3 if ln.gemm2 is not None else 2 if ln.pair else 1
                d.smem_bytes = GEMM_PAIR_SMEM if ln.pair else GEMM_SMEM
                d.a = _operand_desc(ln.gemm[0], lowering, offsets, 128)
                d.b = _operand_desc(ln.gemm[1], lowering, offsets, 128 if ln.pair else 256)
                if ln.gemm2 is not None:
                    d.a2 = _operand_desc(ln.gemm2[0], lowering, offsets, 128)
                    d.b2 = _operand_desc(ln.gemm2[1], lowering, offsets, 128)
                if ln.counters is not None:
                    # a chain's row-block counters or a K split's region counters
                    d.counter_offset = offsets[ln.counters]
                    d.counter_bytes = ln.counter_bytes
            else:
                d.is_gemm = 0
                d.smem_bytes = max(0, ln.smem)
            launches.append(d)
    module = GeneratedModule(
        source=source,
        arena_bytes=max(plan.arena_bytes, 256),
        input_names=list(lowering.inputs),
        output_names=list(lowering.outputs),
        steps=steps,
        offsets=offsets,
        launches=launches,
    )
    return optimised, order, plan, module, lowering


def _tma_ok(gemm) -> bool:
    return all((op.cols * op.elem_bytes) % 16 == 0 for op in gemm)


# ----------------------------------------------------------------------------- compiled graph


class CompiledGraph:
    """A graph compiled for one CUDA device (the counterpart of executor.CompiledGraph)."""

    def __init__(self, graph, order, plan, module: GeneratedModule, lowering: Lowering, device: int):
        import torch

        self.graph = graph
        self.order = list(order)
        self.plan = plan
        self.module = module
        self.lowering = lowering
        self.device = device
        self.input_names = list(module.input_names)
        self._torch = torch
        lib = _lib.load()
        _lib.ensure_device(device)
        with torch.cuda.device(device):
            cubin = compile_source(module.source)
            self._cubin = cubin
            mod = ctypes.c_void_p()
            _lib.check(lib.tgcb_module_load(cubin, len(cubin), ctypes.byref(mod)), "loading the generated module")
            self._module = mod
            arr = (_lib.LaunchDesc * max(1, len(module.launches)))(*module.launches)
            plan_h = ctypes.c_void_p()
            _lib.check(
                lib.tgcb_plan_create(mod, arr, len(module.launches), module.arena_bytes, ctypes.byref(plan_h)),
                "binding the launch plan",
            )
            self._plan = plan_h
            _lib.check(lib.tgcb_plan_set_input_count(plan_h, len(self.input_names)), "declaring the plan's inputs")
        self._out_specs = []
        for name in module.output_names:
            v = lowering.values[name]
            self._out_specs.append((name, v.shape.ints(), _torch_dtype(v.dtype), v.bytes))
        self._in_specs = []
        for name in self.input_names:
            v = lowering.values[name]
            self._in_specs.append((name, v.shape.ints(), _torch_dtype(v.dtype), v.bytes))
        self.function: Callable = self._run
        self.launches_per_call = len(module.launches)

    def close(self) -> None:
        """Release the plan and the module. The module's code is released only after the
        launches of this graph's last calls have finished (tgcb_module_unload waits for the
        events those calls recorded on their streams, not for the whole device); raises
        ``DeviceError`` if that wait fails, in which case the code stays loaded."""
        lib = _lib.load()
        plan, self._plan = getattr(self, "_plan", None), None
        if plan:
            lib.tgcb_plan_destroy(plan)
        module, self._module = getattr(self, "_module", None), None
        if module:
            _lib.check(lib.tgcb_module_unload(module), "unloading the generated module")

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - nothing can be raised from a finaliser
            pass

    @property
    def arena_bytes(self) -> int:
        return self.module.arena_bytes

    def new_arena(self):
        """A fresh device arena of the planned size (256-byte aligned by the caching allocator)."""
        return self._torch.empty(self.arena_bytes, dtype=self._torch.uint8, device=f"cuda:{self.device}")

    def __call__(self, feeds: dict) -> list:
        missing = [n for n in self.input_names if n not in feeds]
        if missing:
            raise ConfigError(f"no value supplied for {missing}")
        return self.function(self.new_arena(), feeds)

    def input_pointers(self, arena, feeds: dict, stream=None) -> list[int]:
        """Device address of each input: the caller's buffer when usable in place, else its slot."""
        torch = self._torch
        base = arena.data_ptr()
        ptrs = []
        for name, shape, dtype, nbytes in self._in_specs:
            t = feeds[name]
            usable = (
                isinstance(t, torch.Tensor)
                and t.is_cuda
                and t.device.index == self.device
                and t.dtype == dtype
                and tuple(t.shape) == tuple(shape)
                and t.is_contiguous()
                and t.data_ptr() % 256 == 0
            )
            if usable:
                ptrs.append(t.data_ptr())
                continue
            off = self.module.offsets[name]
            slot = arena[off : off + nbytes].view(dtype).view(shape) if nbytes else arena[off:off].view(dtype)
            src = t if isinstance(t, torch.Tensor) else torch.as_tensor(t)
            slot.copy_(src.broadcast_to(shape), non_blocking=True)
            ptrs.append(base + off)
        return ptrs

    def _run(self, arena, feeds: dict, stream=None) -> list:
        torch = self._torch
        if arena.numel() < self.arena_bytes or not arena.is_cuda:
            raise ConfigError(f"the arena needs {self.arena_bytes} device bytes")
        missing = [n for n in self.input_names if n not in feeds]
        if missing:
            raise ConfigError(f"no value supplied for {missing}")
        with torch.cuda.device(self.device):
            s = stream if stream is not None else torch.cuda.current_stream(self.device)
            with torch.cuda.stream(s):  # input copies are ordered before the kernels that read them
                ptrs = self.input_pointers(arena, feeds)
            arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
            rc = _lib.load().tgcb_plan_run(self._plan, ctypes.c_void_p(arena.data_ptr()), arr, len(ptrs), ctypes.c_void_p(s.cuda_stream))
            _lib.check(rc, "running the compiled graph")
            return self._outputs(arena, feeds)

    def run_range(self, arena, ptrs: list[int], first: int, count: int, stream) -> None:
        """Queue launches [first, first+count) on ``stream`` with input addresses from ``input_pointers``."""
        arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
        rc = _lib.load().tgcb_plan_run_range(
            self._plan, first, count, ctypes.c_void_p(arena.data_ptr()), arr, len(ptrs), ctypes.c_void_p(stream.cuda_stream)
        )
        _lib.check(rc, "running part of the compiled graph")

    def launch_writers(self) -> dict[str, int]:
        """For every materialised value, the index of the last launch of the step that writes it."""
        out: dict[str, int] = {}
        k = 0
        for s in self.module.steps:
            k += len(s.launches)
            for w in s.writes:
                out[w] = k - 1
        return out

    def run_profiled(self, arena, feeds: dict, stream=None) -> tuple[list, list[float]]:
        """Run once with a CUDA event around every launch; returns (outputs, ms per launch).

        Waits for the stream. The events are recorded on the stream the kernels run on.
        """
        torch = self._torch
        with torch.cuda.device(self.device):
            s = stream if stream is not None else torch.cuda.current_stream(self.device)
            with torch.cuda.stream(s):
                ptrs = self.input_pointers(arena, feeds)
            arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
            n = len(self.module.launches)
            ms = (ctypes.c_float * max(1, n))()
            rc = _lib.load().tgcb_plan_run_profiled(
                self._plan, ctypes.c_void_p(arena.data_ptr()), arr, len(ptrs), ctypes.c_void_p(s.cuda_stream), ms
            )
            _lib.check(rc, "running the compiled graph (profiled)")
            return self._outputs(arena, feeds), [float(ms[i]) for i in range(n)]

    def _outputs(self, arena, feeds: dict) -> list:
        outs = []
        for name, shape, dtype, nbytes in self._out_specs:
            if name in self.input_names:
                outs.append(feeds[name].to(device=arena.device, dtype=dtype).clone())
                continue
            off = self.module.offsets[name]
            outs.append(arena[off : off + nbytes].view(dtype).view(shape))
        return outs

    def check_status(self) -> None:
        """Synchronise and raise ``DeviceError`` if any kernel recorded a device-side failure."""
        st = ctypes.c_int(0)
        _lib.check(_lib.load().tgcb_status(1, ctypes.byref(st)), "reading the device status")
        if st.value != 0:
            raise DeviceError(f"a kernel reported device status {st.value} (timeout or bad launch)")

    def as_dict(self) -> dict:
        return {
            "nodes": len(self.graph.nodes),
            "arena_bytes": self.arena_bytes,
            "generated_lines": self.module.lines,
            "kernels": len(self.module.launches),
            "steps": [s.kind for s in self.module.steps],
        }


def compile_graph(graph, *, pipeline=None, optimise: bool = True, device: int | None = None) -> CompiledGraph:
    """Optimise, schedule, partition, allocate and compile ``graph`` for a B200 (cf. executor.py:91-122)."""
    import torch

    if not torch.cuda.is_available():
        raise DeviceError("compile_graph needs a CUDA device; the B200 backend has no CPU path")
    dev = torch.cuda.current_device() if device is None else device
    optimised, order, plan, module, lowering = generate(graph, pipeline=pipeline, optimise=optimise)
    return CompiledGraph(optimised, order, plan, module, lowering, dev)


def delay(ns: int, stream=None) -> None:
    """Queue a bounded spin kernel (at most 10 ms) so launches queued behind it start back to back."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(_lib.load().tgcb_delay(int(ns), ctypes.c_void_p(s.cuda_stream)), "tgcb_delay")


def source_of(graph) -> str:
    """The generated CUDA for a graph, without a device (cf. executor.source_of)."""
    return generate(graph)[3].source
