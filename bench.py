#!/usr/bin/env python
"""Benchmark of the B200 backend on tgc's workloads; prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tgcb|reference] [--workload NAME]

Default workload ``mlp``: the transformer MLP block (layernorm -> x@W1+b1 -> tanh-form GELU
-> @W2+b2; x [8192,1024], W1 [1024,4096], W2 [4096,1024], fp32 with TF32 tensor-core GEMMs),
compiled by ``tgcb.runtime.compile_graph`` from tgc's graph and run as three kernels. A
step is one execution of the compiled graph. Other workloads: ``cone`` (x [4096,1024] ->
exp -> three row reductions), ``int8`` (per-token/per-channel int8 linear
8192x4096x4096), ``longsum`` (bit-exact pairwise sum of 2^26 floats).

Multi-GPU (torchrun, one process per GPU, NCCL): for the forward workloads every rank runs
its own shard of rows, so work per GPU is fixed ("weak") and ``value`` = executions by all
ranks / the slowest rank's device time; ``train`` splits one 65536-row global batch over the
ranks ("strong") and averages the gradients with NCCL, one unit being one global step. Timing: W warm-up steps; then K steps, each timed with CUDA events recorded on
the stream the kernels run on (one event around every kernel, tgcb_plan_run_profiled); L2
flushed before every timed step outside the events (a 256 MiB write, then a 256 MiB read so
the flush leaves no dirty lines to be written back inside a timed kernel); a bounded delay
kernel queued ahead of each step so its launches start back to back; barrier + synchronize
on both sides; the max over ranks.

``e2e`` times the same step through the public API with host buffers: every step copies all
inputs from pinned host memory into the arena and reads the results back to pinned host
memory inside the timed region.

``--impl reference`` times tgc's own CPU path restated by oracle/ (the generated-Python
executor: one torch CPU op per node into one arena) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "tensor-graph-compiler_b200"))
sys.path.insert(0, REPO)

METRIC = "fused-graph execs/sec and achieved HBM GB/s (% of peak) at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
L2_NOTE = (
    "flushed before every timed step: 256 MiB write, then a 256 MiB read so no dirty flush "
    "lines are written back inside the timed kernels"
)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["tgcb", "reference"], default="tgcb")
    p.add_argument("--workload", choices=["mlp", "cone", "int8", "longsum", "train", "attention"], default="mlp")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--only", action="store_true", help="time the chosen workload alone, without the others under 'workloads'")
    p.add_argument("--sub-steps", type=int, default=0, help="timed steps of each nested workload (default: --steps)")
    p.add_argument("--train-rows", type=int, default=65536, help="global batch of the train workload (profiling uses a small one)")
    p.add_argument("--train-buckets", choices=["final", "per_gradient", "two", "peer"], default="peer",
                   help="train: one grouped gradient all-reduce after the backward, or one per gradient as it becomes final")
    p.add_argument("--train-side-ctas", type=int, default=20,
                   help="train with two buckets: CTA limit of the communicator that runs the early bucket")
    return p.parse_args()


def peaks() -> tuple[dict, str]:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi queried every 200 ms (read-only); summarises the samples of the timed region.

    Started before the warm-up so sampling is running when timing begins; ``mark_start`` and
    ``mark_end`` bracket the timed region in wall time. The samples inside it, plus the
    nearest one on each side (a region shorter than the period still gets readings), are
    summarised.
    """

    FIELDS = (
        "timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t0 = self.t1 = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
            return
        first = threading.Event()

        def reader():
            for line in self.proc.stdout:
                self.lines.append((time.time(), line.strip()))
                first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        first.wait(timeout=10)

    def mark_start(self) -> None:
        self.t0 = time.time()

    def mark_end(self) -> None:
        self.t1 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        t0, t1 = self.t0 or 0.0, self.t1 or time.time()
        inside = [ln for ts, ln in self.lines if t0 <= ts <= t1]
        before = [ln for ts, ln in self.lines if ts < t0][-1:]
        after = [ln for ts, ln in self.lines if ts > t1][:1]
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in before + inside + after:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9], strict=True):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {
            "sm_mhz": statistics.median(sm),
            "sm_max_mhz": max(mx),
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "samples_inside_timed_region": len(inside),
            "reasons": sorted(reasons),
        }


class NvmlClockSampler:
    """NVML read every millisecond in a thread (read-only queries of the SM clock, its maximum,
    power and the active clock-event reasons); summarises the samples of the timed region.

    The timed regions here last milliseconds, well under nvidia-smi's shortest period, so the
    same readings nvidia-smi reports are taken directly from NVML for the GPU this rank drives
    (matched by UUID). Falls back to ``ClockSampler`` when NVML is unavailable.
    """

    def __init__(self, local: int):
        self.local = local
        self.samples: list[tuple[float, float, float, float, int]] = []
        self.t0 = self.t1 = None
        self.stop_flag = threading.Event()

    def start(self) -> bool:
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.local).uuid)
            try:
                h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except pynvml.NVMLError:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.local)
            self.nvml, self.h = pynvml, h
            self.max_sm = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - any NVML failure means: use nvidia-smi instead
            return False

        def poll():
            p = self.nvml
            while not self.stop_flag.is_set():
                try:
                    self.samples.append((
                        time.time(),
                        float(p.nvmlDeviceGetClockInfo(self.h, p.NVML_CLOCK_SM)),
                        self.max_sm,
                        p.nvmlDeviceGetPowerUsage(self.h) / 1000.0,
                        int(p.nvmlDeviceGetCurrentClocksEventReasons(self.h)),
                    ))
                except p.NVMLError:
                    pass
                time.sleep(0.001)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        return True

    def mark_start(self) -> None:
        self.t0 = time.time()

    def mark_end(self) -> None:
        self.t1 = time.time()

    def stop(self) -> dict:
        time.sleep(0.01)
        self.stop_flag.set()
        self.thread.join(timeout=5)
        p = self.nvml
        t0, t1 = self.t0 or 0.0, self.t1 or time.time()
        inside = [x for x in self.samples if t0 <= x[0] <= t1]
        use = inside or ([x for x in self.samples if x[0] < t0][-1:] + [x for x in self.samples if x[0] > t1][:1])
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": "nvml"}
        bits = {
            "hw_slowdown": p.nvmlClocksEventReasonHwSlowdown,
            "hw_thermal_slowdown": p.nvmlClocksEventReasonHwThermalSlowdown,
            "sw_thermal_slowdown": p.nvmlClocksEventReasonSwThermalSlowdown,
            "sw_power_cap": p.nvmlClocksEventReasonSwPowerCap,
        }
        reasons = sorted({name for x in use for name, b in bits.items() if x[4] & b})
        return {
            "sm_mhz": statistics.median(x[1] for x in use),
            "sm_max_mhz": max(x[2] for x in use),
            "sm_mhz_min": min(x[1] for x in use),
            "power_w_max": round(max(x[3] for x in use), 1),
            "samples": len(use),
            "samples_inside_timed_region": len(inside),
            "reasons": reasons,
            "source": "nvml, 1 ms period",
        }


# ----------------------------------------------------------------------------- workloads


def library_gemm_reference(runner, shapes, steps: int, int8: bool = False) -> dict:
    """cuBLAS (through torch) on the same GEMM shapes, timed the same way (L2 flushed, events
    around each call): a like-for-like library reference for the tensor-core kernels, not part
    of any measured step. TF32 for float32 (torch.mm with TF32 allowed), int8 x int8 -> int32
    (torch._int_mm) for int8."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    out = {}
    try:
        for name, (m, k, n) in shapes.items():
            if int8:
                a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=runner.device)
                b = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=runner.device).t()  # [k, n], K-major
                fn = lambda a=a, b=b: torch._int_mm(a, b)  # noqa: E731
            else:
                a = torch.randn(m, k, device=runner.device)
                b = torch.randn(k, n, device=runner.device)
                c = torch.empty(m, n, device=runner.device)
                fn = lambda a=a, b=b, c=c: torch.mm(a, b, out=c)  # noqa: E731

            def step(fn=fn):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                e.synchronize()
                return [s.elapsed_time(e)]

            for _ in range(3):
                step()
            ms = runner.timed(step, steps)[0] / steps
            rate = 2.0 * m * k * n / (ms * 1e-3) / 1e12
            out[name] = {"shape_mkn": [m, k, n], "us": round(ms * 1e3, 2), ("TOP/s" if int8 else "TFLOP/s"): round(rate, 1)}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    out["what"] = ("cuBLAS through torch (" + ("torch._int_mm, int32 output only" if int8 else "torch.mm, TF32, no epilogue")
                   + "), same flush and event discipline as the measured steps; a library reference, not a step")
    return out


class GraphWorkload:
    """A workload that is one tgc graph compiled by tgcb.runtime.compile_graph."""

    name = ""
    unit = "execs/s"
    dtype = ""

    def __init__(self, rank: int):
        self.rank = rank

    def graph(self):
        raise NotImplementedError

    def feeds(self) -> dict:
        raise NotImplementedError

    def config(self) -> dict:
        raise NotImplementedError

    def setup(self, device) -> None:
        import torch

        from tgcb.runtime import compile_graph

        self.g = self.graph()
        self.compiled = compile_graph(self.g, device=device.index)
        self.cpu_feeds = self.feeds()
        self.dev_feeds = {k: v.to(device) for k, v in self.cpu_feeds.items()}
        self.host_feeds = {k: v.pin_memory() for k, v in self.cpu_feeds.items()}
        self.arena = self.compiled.new_arena()
        self.out_host = [
            torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in self.compiled.function(self.arena, self.dev_feeds)
        ]
        torch.cuda.synchronize()
        self.compiled.check_status()

    def launches_per_step(self) -> int:
        return self.compiled.launches_per_call

    def step_profiled(self) -> list[float]:
        return self.compiled.run_profiled(self.arena, self.dev_feeds)[1]

    def step_e2e(self) -> None:
        outs = self.compiled.function(self.arena, self.host_feeds)
        for o, h in zip(outs, self.out_host, strict=True):
            h.copy_(o, non_blocking=True)

    def run_e2e(self, steps: int) -> float:
        """``steps`` calls of the public API from pinned host feeds to pinned host results,
        alternating two streams and two arenas so one call's copies overlap the next call's
        (every call still copies all of its inputs in and all of its outputs out). Device time
        from an event before the first call to one after the last, in ms."""
        import torch

        if not hasattr(self, "arena2"):
            self.arena2 = self.compiled.new_arena()
            self.out_host2 = [torch.empty_like(h).pin_memory() for h in self.out_host]
            self.streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        arenas, hosts = (self.arena, self.arena2), (self.out_host, self.out_host2)
        cur = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(cur)
        for st in self.streams:
            st.wait_event(start)
        for i in range(steps):
            st = self.streams[i % 2]
            with torch.cuda.stream(st):
                outs = self.compiled.function(arenas[i % 2], self.host_feeds, stream=st)
                for o, h in zip(outs, hosts[i % 2], strict=True):
                    h.copy_(o, non_blocking=True)
        for st in self.streams:
            cur.wait_stream(st)
        end.record(cur)
        end.synchronize()
        return start.elapsed_time(end)

    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.host_feeds.values())

    def d2h_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.out_host)

    def kernel_work(self) -> list[dict]:
        """Per launch: name, kind, roofline bound and algorithmic work (bytes or ops)."""
        low = self.compiled.lowering
        out = []
        for s in self.compiled.module.steps:
            if s.kind == "gemm":
                # one GEMM, or a chain of two in one launch (label "first+second")
                work = 0
                for label in s.label.split("+"):
                    node = low.producers[label]
                    M, K = low.sizes(node.inputs[0])
                    N = low.sizes(node.inputs[1])[1]
                    is_int = node.output.dtype.name == "int32"
                    work += 2 * M * N * K
                # a chain launch may also compute its first GEMM's A rows (a row prologue); those
                # bytes are not in the tensor-bound work
                rows = [n for n in s.nodes if n in low.producers and low.producers[n].op.category == "reduction"]
                also = (f"computes the rows of {', '.join(rows)} (row prologue) besides the GEMM FLOPs counted in achieved"
                        if rows else None)
                for ln in s.launches:
                    out.append({"name": ln.kernel, "kind": s.kind, "bound": "tensor", "work": work,
                                "type": "int8" if is_int else "tf32", "also": also})
                continue
            rbytes = sum(low.values[r].bytes for r in s.reads if r in low.values)
            wbytes = sum(low.values[w].bytes for w in s.writes if w in low.values)
            for i, ln in enumerate(s.launches):
                out.append({"name": ln.kernel, "kind": s.kind, "bound": "hbm", "work": rbytes + wbytes if i == 0 else 0})
        return out

    def cpu_program(self):
        from oracle import interp

        return interp.generated_python_program(self.g)


class MlpWorkload(GraphWorkload):
    name = "mlp"
    dtype = "tf32"
    machine_kind = "tf32"
    rows = 8192

    def graph(self):
        from tgcb import ir, workloads

        return workloads.mlp_graph(ir.Builder, rows=self.rows)

    def feeds(self):
        from tgcb import workloads

        return workloads.mlp_inputs(rows=self.rows, seed=self.rank)

    def extras(self, runner, steps: int) -> dict:
        ref = library_gemm_reference(runner, {"gemm1": (self.rows, 1024, 4096), "gemm2": (self.rows, 4096, 1024)}, steps)
        if runner.rank != 0:
            return {}
        ref["gemm1_plus_gemm2_us"] = round(ref["gemm1"]["us"] + ref["gemm2"]["us"], 2)
        return {"library_reference": ref}

    def config(self):
        return {
            "workload": "transformer MLP block: layernorm(gamma=1,beta=0) -> x@W1+b1 -> GELU(tanh form) -> @W2+b2; "
            "x [8192,1024] ~N(0,1), W1 [1024,4096], W2 [4096,1024] ~N(0,0.02), zero biases; fp32 graph, TF32 GEMMs",
            "rows_per_gpu": self.rows,
            "flops_per_exec": 2 * self.rows * 1024 * 4096 * 2,
            "l2": L2_NOTE,
        }


class ConeWorkload(GraphWorkload):
    name = "cone"
    dtype = "f32"
    machine_kind = "fp32"

    def graph(self):
        from tgcb import ir, workloads

        return workloads.cone_graph(ir.Builder)

    def feeds(self):
        from tgcb import workloads

        return workloads.cone_inputs(seed=self.rank)

    def config(self):
        return {
            "workload": "fused cone: t=exp(0.5*x-1) over x [4096,1024] fp32 ~N(0,1); row-sum(t), row-max(t), row-sum(t*x)",
            "bytes_per_exec": 4096 * 1024 * 4 + 3 * 4096 * 4,
            "l2": L2_NOTE,
        }

    def extras(self, runner, steps: int) -> dict:
        """The launch's ceiling, the outputs' error against float64, and tgc's fusion plans.

        Ceiling: the same launch shape reading the same 16 MiB and only adding it up (a row sum
        over x, compiled by the same codegen), timed the same way; what any kernel over these
        bytes in one launch reaches here. Errors: each output's largest relative difference
        from the same computation in float64 (torch, on the GPU). Plans: tgc's fusion search
        (tgcb.fusion_search) on this graph, every strategy priced by tgc's rules and turned into
        time on the B200 roofline, beside the backend's one-pass kernel.
        """
        import torch

        from tgcb import cost, fusion_search, ir, workloads
        from tgcb.runtime import compile_graph

        ceiling = compile_graph(workloads.row_sum_graph(ir.Builder), device=runner.device.index)
        arena = ceiling.new_arena()
        feeds = {"x": self.dev_feeds["x"]}
        for _ in range(3):
            ceiling.run_profiled(arena, feeds)
        ceiling_ms = runner.max_over_ranks(sum(runner.timed(lambda: ceiling.run_profiled(arena, feeds)[1], steps))) / steps
        cone_ms = runner.max_over_ranks(sum(runner.timed(self.step_profiled, steps))) / steps
        outs = self.compiled.function(self.arena, self.dev_feeds)
        x = self.dev_feeds["x"].double()
        t = torch.exp(x * 0.5 + (-1.0))
        ref = (t.sum(1), t.amax(1), (t * x).sum(1))
        names = ("row_sum", "row_max", "row_sum_tx")
        errors = {k: float(((o.double() - r).abs() / r.abs()).max()) for k, o, r in zip(names, outs, ref, strict=True)}
        if runner.rank != 0:
            return {}
        machine = cost.b200(runner.peaks, "fp32")
        dag, _ = fusion_search.dag_of(self.g)
        plans = []
        for row in fusion_search.compare(dag):
            plan = fusion_search.FusionPlan(frozenset(row["materialised"]), row["groups"], row["flops"], row["traffic"])
            secs = fusion_search.predicted_seconds(plan, machine.flops_per_second, machine.bytes_per_second)
            plans.append({**{k: row[k] for k in ("strategy", "groups", "flops", "traffic", "cost")},
                          "predicted_us": round(secs * 1e6, 3)})
        best_tgc = min((p for p in plans if not p["strategy"].startswith("one pass")), key=lambda p: p["cost"])
        one = next(p for p in plans if p["strategy"].startswith("one pass"))
        return {
            "ceiling": {
                "kernel": "tgcb_row_1 of row_sum over the same x (same grid, block and bytes; only adds)",
                "ceiling_us": round(ceiling_ms * 1e3, 2),
                "cone_us": round(cone_ms * 1e3, 2),
                "cone_over_ceiling": round(ceiling_ms / cone_ms, 4),
                "ceiling_gbs": round(16 * 2**20 / (ceiling_ms * 1e-3) / 1e9, 1),
                "note": "both timed back to back here with L2 flushed; a 16 MiB launch is bound by launch ramp and "
                        "drain, not by HBM (64 MiB and 256 MiB reads reach higher fractions)",
            },
            "error_vs_fp64": {**{k: {"max_rel_error": v} for k, v in errors.items()},
                              "declared_bracketing": "row tree (tgcb_row_1): bit-exact to oracle/bracketing.c "
                                                     "oracle_row_tree in the GPU tests, i.e. zero error against the "
                                                     "chosen bracketing"},
            "fusion_search": {
                "machine": machine.as_dict(),
                "plans": plans,
                "best_tgc_plan": best_tgc["strategy"],
                "predicted_speedup_of_one_pass_over_best_tgc_plan": round(best_tgc["predicted_us"] / one["predicted_us"], 3),
                "model_cost_regret_of_best_tgc_plan": round(best_tgc["cost"] / one["cost"], 4),
            },
        }


class Int8Workload(GraphWorkload):
    """The int8 linear layer as a serving step: the float32 activations are quantised per token
    on the GPU (tgcb.quantize, bit-exact to tgc's per_row_schemes + quantise), then the
    compiled graph runs the int8 GEMM with int32 accumulation and the fused dequantisation.
    The weight is quantised per output channel once, outside the step (tgc hoists it the same
    way: passes/hoisting.py)."""

    name = "int8"
    dtype = "int8 x int8 -> int32, f32 dequant"
    machine_kind = "int8"
    rows, k, n = 8192, 4096, 4096

    def graph(self):
        from tgcb import ir, workloads

        return workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32)

    def feeds(self):
        """Host-side inputs for the CPU restatement: float32 activations, quantised weight."""
        import torch

        from oracle import quantize as oq
        from tgcb import workloads

        ins = workloads.int8_inputs(seed=self.rank)
        qwt, sw = oq.quantise_rows(ins["w"].T.contiguous().numpy())
        return {"a": ins["a"], "qwt": torch.from_numpy(qwt), "sw": torch.from_numpy(sw).reshape(1, -1)}

    def config(self):
        return {"workload": "int8 linear: A [8192,4096] f32 quantised per token on the GPU -> qa x qwt^T [4096,4096] "
                            "-> int32 acc -> *sa *sw (f32); W quantised once outside the step",
                "int_ops_per_exec": 2 * self.rows * self.k * self.n, "l2": L2_NOTE}

    def setup(self, device) -> None:
        import torch

        from tgcb import quantize, workloads
        from tgcb.runtime import compile_graph

        self.g = self.graph()
        self.compiled = compile_graph(self.g, device=device.index)
        ins = workloads.int8_inputs(seed=self.rank)
        self.a_host = ins["a"].pin_memory()
        self.a_dev = ins["a"].to(device)
        qwt, sw = quantize.quantise_rows(ins["w"].T.contiguous().to(device))
        self.weights = {"qwt": qwt, "sw": sw.reshape(1, -1)}
        self.sets = []
        for _ in range(2):  # two independent buffer sets for the pipelined end-to-end run
            qa = torch.empty(self.rows, self.k, dtype=torch.int8, device=device)
            sa = torch.empty(self.rows, dtype=torch.float32, device=device)
            self.sets.append({"a": torch.empty_like(self.a_dev), "qa": qa, "sa": sa, "arena": self.compiled.new_arena(),
                              "feeds": {"qa": qa, "sa": sa.reshape(-1, 1), **self.weights}})
        self.arena = self.sets[0]["arena"]
        quantize.quantise_rows_into(self.a_dev, self.sets[0]["qa"], self.sets[0]["sa"])
        outs = self.compiled.function(self.arena, self.sets[0]["feeds"])
        self.out_host = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
        self.out_host2 = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
        torch.cuda.synchronize()
        self.compiled.check_status()

    @property
    def cpu_feeds(self):
        if not hasattr(self, "_cpu_feeds"):
            self._cpu_feeds = self.feeds()
        return self._cpu_feeds

    @cpu_feeds.setter
    def cpu_feeds(self, value):
        self._cpu_feeds = value

    def launches_per_step(self) -> int:
        return 1 + self.compiled.launches_per_call

    def step_profiled(self) -> list[float]:
        import torch

        from tgcb import quantize

        st = self.sets[0]
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        quantize.quantise_rows_into(self.a_dev, st["qa"], st["sa"])
        e.record()
        ms = self.compiled.run_profiled(st["arena"], st["feeds"])[1]
        return [s.elapsed_time(e)] + ms

    def _e2e_call(self, st, out_host, stream) -> None:
        from tgcb import quantize

        st["a"].copy_(self.a_host, non_blocking=True)
        quantize.quantise_rows_into(st["a"], st["qa"], st["sa"], stream=stream)
        outs = self.compiled.function(st["arena"], st["feeds"], stream=stream)
        for o, h in zip(outs, out_host, strict=True):
            h.copy_(o, non_blocking=True)

    def step_e2e(self) -> None:
        import torch

        self._e2e_call(self.sets[0], self.out_host, torch.cuda.current_stream())

    def run_e2e(self, steps: int) -> float:
        """As GraphWorkload.run_e2e: float32 activations in from pinned host memory, quantised,
        multiplied and dequantised, both outputs back to pinned host memory, alternating two
        streams and two buffer sets."""
        import torch

        if not hasattr(self, "streams"):
            self.streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        cur = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(cur)
        for st in self.streams:
            st.wait_event(start)
        for i in range(steps):
            st = self.streams[i % 2]
            with torch.cuda.stream(st):
                self._e2e_call(self.sets[i % 2], self.out_host if i % 2 == 0 else self.out_host2, st)
        for st in self.streams:
            cur.wait_stream(st)
        end.record(cur)
        end.synchronize()
        return start.elapsed_time(end)

    def h2d_bytes(self) -> int:
        return self.a_host.numel() * 4

    def extras(self, runner, steps: int) -> dict:
        ref = library_gemm_reference(runner, {"gemm": (self.rows, self.k, self.n)}, steps, int8=True)
        return {"library_reference": ref} if runner.rank == 0 else {}

    def kernel_work(self) -> list[dict]:
        quant = self.rows * self.k * 4 + self.rows * self.k + self.rows * 4
        return [{"name": "quantise_rows_i8", "kind": "quantise", "bound": "hbm", "work": quant}] + GraphWorkload.kernel_work(self)

    def cpu_program(self):
        from oracle import interp
        from oracle import quantize as oq

        g = self.g

        def run(feeds):
            qa, sa = oq.quantise_rows(feeds["a"].numpy())
            import torch

            return interp.run(g, {"qa": torch.from_numpy(qa), "sa": torch.from_numpy(sa).reshape(-1, 1),
                                  "qwt": feeds["qwt"], "sw": feeds["sw"]})

        return run


class LongSumWorkload:
    """Pairwise (block 8) float32 sum of 2^26 values per GPU, bit-exact to tgc's summation.pairwise.

    On N GPUs the vector is N * 2^26 values long and each rank holds one depth-log2(N) subtree
    of the halving; a step sums the rank's slice with the same kernels, all-gathers the N
    partials (one float each, NCCL) and combines them by the perfect tree of the top levels, so
    every rank ends with the whole vector's bit-exact sum. Work per GPU is fixed ("weak"); one
    unit is 2^26 values summed.
    """

    name = "longsum"
    unit = "sums/s"
    dtype = "f32"
    n = 1 << 26

    def __init__(self, rank: int):
        self.rank = rank
        self.world = 1

    def config(self):
        return {"workload": "pairwise (block 8) sum of 2^26 fp32 values ~U(0,1) with one 1e8 entry per GPU; "
                            "on N GPUs one sum of the N * 2^26-value vector per step",
                "bytes_per_sum": self.n * 4, "l2": L2_NOTE}

    def parallelism(self, n: int) -> str:
        if n == 1:
            return "dp1: one 2^26-value sum"
        return (f"dp{n}: each GPU sums its 2^26-value subtree, NCCL all-gather of {n} partials, "
                "perfect-tree combine of the top levels on every GPU")

    def setup(self, device, dist=None, world: int = 1):
        import torch

        from tgcb import summation, workloads

        self.world = world
        self.v, _ = workloads.longsum_input(self.n, seed=self.rank)
        self.dev = self.v.to(device)
        self.host = self.v.pin_memory()
        self.out = torch.empty(1, dtype=torch.float32, device=device)
        self.out_host = torch.empty(1, dtype=torch.float32).pin_memory()
        self.scratch = torch.empty(summation.scratch_bytes(self.n), dtype=torch.uint8, device=device)
        self.staging = torch.empty_like(self.dev)
        self.sharded = None
        if world > 1:
            self.sharded = summation.ShardedPairwise(self.n * world, self.rank, world, dist, device)
            self.partial = torch.empty(1, dtype=torch.float32, device=device)

    def launches_per_step(self) -> int:
        # the leaf kernel and its dependent final block; on N GPUs also the top-level tree
        # (the all-gather is NCCL's kernel, not counted)
        return 2 if self.world == 1 else 3

    def step_profiled(self) -> list[float]:
        import torch

        from tgcb import summation

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        if self.sharded is None:
            ev[0].record()
            summation.pairwise_into(self.dev, self.out, self.scratch)
            ev[1].record()
            ev[1].synchronize()
            return [ev[0].elapsed_time(ev[1])]
        ev[0].record()
        summation.pairwise_into(self.dev, self.sharded.partial, self.scratch)
        ev[1].record()
        self.sharded.dist.all_gather_into_tensor(self.sharded.gathered, self.sharded.partial)
        summation.perfect_tree_into(self.sharded.gathered, self.out)
        ev[2].record()
        ev[2].synchronize()
        return [ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])]

    def extras(self, runner, steps: int) -> dict:
        """The sequential schedule's latency, and both schedules' error against float64.

        Sequential: one chain of 2^26 dependent additions, so its time is latency, not
        bandwidth; timed 3 times (L2 flushed). Errors: on this rank's 2^26-value vector (rank 0
        holds the seed-0 vector of the long-sum workload), the pairwise and sequential results
        against the correctly rounded float64 sum (tgcb.summation.exact, tgc's summation.exact).
        """
        import torch

        from tgcb import summation

        seq_out = torch.empty(1, dtype=torch.float32, device=runner.device)
        pw_out = torch.empty(1, dtype=torch.float32, device=runner.device)

        def seq_step():
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            summation.sequential_into(self.dev, seq_out)
            e.record()
            e.synchronize()
            return [s.elapsed_time(e)]

        seq_step()
        seq_ms = runner.max_over_ranks(runner.timed(seq_step, 3)[0]) / 3
        summation.pairwise_into(self.dev, pw_out, self.scratch)
        torch.cuda.synchronize()
        if runner.rank != 0:
            return {}
        exact = summation.exact(self.dev)
        pw, sq = float(pw_out.item()), float(seq_out.item())
        return {
            "sequential": {
                "ms": round(seq_ms, 3),
                "gbs": round(self.n * 4 / (seq_ms * 1e-3) / 1e9, 2),
                "bound": "latency: one chain of 2^26 dependent float adds on one thread",
                "kernel": "sequential_staged",
            },
            "error_vs_fp64": {
                "vector": "rank 0's 2^26 values (the long-sum workload's seed-0 input)",
                "exact_fp64": exact,
                "pairwise": {"value": pw, "rel_error": summation.relative_error(pw, exact)},
                "sequential": {"value": sq, "rel_error": summation.relative_error(sq, exact)},
                "declared_bracketing": "both schedules are bit-exact to tgc's summation.pairwise / sequential "
                                       "(tests), i.e. zero error against the chosen bracketing",
            },
        }

    def step_e2e(self) -> None:
        from tgcb import summation

        self.staging.copy_(self.host, non_blocking=True)
        if self.sharded is None:
            summation.pairwise_into(self.staging, self.out, self.scratch)
        else:
            self.sharded.into(self.staging, self.out)
        self.out_host.copy_(self.out, non_blocking=True)

    def h2d_bytes(self) -> int:
        return self.n * 4

    def d2h_bytes(self) -> int:
        return 4

    def kernel_work(self) -> list[dict]:
        work = [{"name": "pairwise_leaves_pdl+pairwise_final", "kind": "longsum", "bound": "hbm", "work": self.n * 4}]
        if self.world > 1:
            work.append({"name": "nccl_all_gather+perfect_tree", "kind": "exchange", "bound": "nvlink", "work": 4 * self.world})
        return work

    def cpu_program(self):
        from oracle import bracketing

        v = self.v.numpy()
        return lambda feeds: bracketing.pairwise(v)

    @property
    def cpu_feeds(self):
        return {}


class TrainWorkload:
    """Reverse-mode step of the MLP block: MSE over a 65536-row global batch, sharded over ranks.

    Each rank runs tgc's gradient graph of its shard (tgcb.grad + compile_graph) and the four
    gradients are averaged with NCCL, each all-reduce starting when its gradient is final.
    Total work is fixed as N grows ("strong"); one unit is one global step.
    """

    name = "train"
    unit = "train steps/s"
    dtype = "tf32"
    machine_kind = "tf32"
    scaling = "strong"
    buckets = "peer"
    side_ctas = 20
    global_rows = 65536
    payload = 2 * 1024 * 4096 * 4 + 4096 * 4 + 1024 * 4

    def __init__(self, rank: int):
        self.rank = rank

    def config(self):
        return {
            "workload": "MLP block training step: d/dW of mean((mlp(x)-target)^2), x,target [65536,1024] batch-sharded, "
            "W1 [1024,4096], W2 [4096,1024]; gradients averaged over the GPUs by an all-reduce",
            "global_rows": self.global_rows,
            "flops_per_step": 5 * 2 * self.global_rows * 1024 * 4096,
            "allreduce_bytes": self.payload,
            "l2": L2_NOTE,
        }

    def units_per_step(self, n: int) -> int:
        return 1

    def setup(self, device, dist=None, world: int = 1):
        import torch

        from tgcb import parallel, workloads

        self.world = world
        self.step_obj = parallel.DataParallelTrainStep(self.global_rows, world, self.rank, dist=dist, device=device,
                                                       buckets=self.buckets, side_ctas=self.side_ctas)
        self.g = self.step_obj.graph
        feeds = workloads.mlp_inputs(rows=self.global_rows, target=True)
        x, t = self.step_obj.shard(feeds["x"], feeds["target"])
        self.cpu_feeds = {**{k: feeds[k] for k in parallel.GRADS}, "x": x.contiguous(), "target": t.contiguous()}
        self.dev_feeds = {k: v.to(device) for k, v in self.cpu_feeds.items()}
        self.host_feeds = {k: v.pin_memory() for k, v in self.cpu_feeds.items()}
        outs = self.step_obj.step(self.dev_feeds)
        self.out_host = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
        torch.cuda.synchronize()
        self.compiled = self.step_obj.compiled

    def launches_per_step(self) -> int:
        # the peer all-reduce adds one kernel per bucket
        extra = 0
        if self.step_obj.peer is not None:
            extra = 2 if self.step_obj.early_outs else 1
        return self.compiled.launches_per_call + extra

    def step_profiled(self) -> list[float]:
        import torch

        main = torch.cuda.current_stream()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        timing = []
        s.record(main)
        self.step_obj.step(self.dev_feeds, timing=timing)
        e.record(main)
        e.synchronize()
        per = [a.elapsed_time(b) for a, b in timing]
        total = s.elapsed_time(e)
        return per + [max(0.0, total - sum(per))]

    def close(self) -> None:
        self.step_obj.close()

    def step_e2e(self) -> None:
        outs = self.step_obj.step(self.host_feeds)
        for o, h in zip(outs, self.out_host, strict=True):
            h.copy_(o, non_blocking=True)

    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.host_feeds.values())

    def d2h_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.out_host)

    def kernel_work(self) -> list[dict]:
        return GraphWorkload.kernel_work(self) + [
            {"name": "gaps between launches" if self.world == 1 else
             "exposed peer all-reduce and gaps" if self.buckets == "peer" else "exposed NCCL all-reduce and gaps",
             "kind": "allreduce", "bound": "nvlink", "work": self.payload}
        ]

    def extras(self, runner, steps: int) -> dict:
        """On 2+ GPUs: the gradient all-reduce alone, measured, beside tgc's all-reduce model.

        The 33,574,912-byte gradient set is all-reduced (NCCL AVG) as one flat buffer, 10 times
        after 3 warm-ups, each event-timed, max over ranks; a one-float all-reduce gives the
        start-up latency. tgc's ring model (tgcb.collective, collective.py:76-379) on an NVLink
        link of the measured 770 GB/s peer-copy bandwidth, with the measured start-up divided
        over the ring's 2(n-1) messages, predicts the same all-reduce, and the four gradients
        reduced one call each.
        """
        import torch

        from tgcb import collective

        n, dist = runner.n, runner.dist
        if n == 1 or dist is None:
            return {}
        flat = torch.zeros(self.payload // 4, dtype=torch.float32, device=runner.device)
        one = torch.zeros(1, dtype=torch.float32, device=runner.device)

        def timed_ar(t, reps):
            for _ in range(3):
                dist.all_reduce(t, op=dist.ReduceOp.AVG)
            total = 0.0
            for _ in range(reps):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                dist.all_reduce(t, op=dist.ReduceOp.AVG)
                e.record()
                e.synchronize()
                total += s.elapsed_time(e)
            return runner.max_over_ranks(total) / reps

        big_ms = timed_ar(flat, 10)
        tiny_ms = timed_ar(one, 10)
        peer_ms = None
        if self.step_obj.peer is not None:
            # the library's own all-reduce over the same four gradients, in a slot of its own
            from tgcb.codegen import NUM_SMS

            outs = self.step_obj.step(self.dev_feeds)
            main = torch.cuda.current_stream()
            for _ in range(3):
                self.step_obj.peer.allreduce_avg(outs, 2, main, NUM_SMS)
            total = 0.0
            for _ in range(10):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(main)
                self.step_obj.peer.allreduce_avg(outs, 2, main, NUM_SMS)
                e.record(main)
                e.synchronize()
                total += s.elapsed_time(e)
            peer_ms = runner.max_over_ranks(total) / 10
            self.step_obj.compiled.check_status()
        if runner.rank != 0:
            return {}
        link = collective.nvlink(latency_seconds=tiny_ms * 1e-3 / (2 * (n - 1)))
        grads = [1024 * 4096 * 4, 4096 * 4, 4096 * 1024 * 4, 1024 * 4]
        return {
            "allreduce": {
                "bytes": self.payload,
                "measured_us": round(big_ms * 1e3, 2),
                "measured_busbw_gbs": round(collective.bus_bandwidth(self.payload, n, big_ms * 1e-3) / 1e9, 1),
                "one_float_us": round(tiny_ms * 1e3, 2),
                "link": link.as_dict(),
                "model_ring_us": round(collective.ring_time(self.payload, n, link) * 1e6, 2),
                "model_tree_us": round(collective.tree_time(self.payload, n, link) * 1e6, 2),
                "model_four_calls_us": round(collective.bucket_time(grads, n, link) * 1e6, 2),
                "model_ring_volume_bytes": collective.ring_volume(self.payload, n),
                "how": "NCCL AVG over one flat buffer of the gradient set's size; the step itself reduces the four "
                       "gradients in one grouped call after the backward",
            }
        } | ({
            "peer_allreduce": {
                "bytes": self.payload,
                "measured_us": round(peer_ms * 1e3, 2),
                "measured_busbw_gbs": round(collective.bus_bandwidth(self.payload, n, peer_ms * 1e-3) / 1e9, 1),
                "how": "tgcb_peer_allreduce_avg_f32 over the four gradients in the step's shared arena, one CTA per SM, "
                       "10 calls after 3 warm-ups, each event-timed, max over ranks",
            }
        } if peer_ms is not None else {})

    def cpu_program(self):
        """One 8192-row shard of the step by the oracle (the full 65536 rows take minutes on a CPU)."""
        from oracle import interp
        from tgcb import parallel, workloads

        g = parallel.train_graph(8192)
        feeds = workloads.mlp_inputs(rows=8192, target=True)
        prog = interp.generated_python_program(g)
        scale = self.global_rows // 8192
        self.cpu_scale = scale
        return lambda _feeds: prog(feeds)


class AttentionWorkload:
    """One head of streaming attention (tgc/analysis/attention.py:97-137): 8192 queries against
    8192 keys and values of width 64, float32, one fused kernel (tgcb.attention). Both products
    run on the CUDA cores in float32, as tgc's float32 matmuls do; the roofline is the CUDA
    cores' nominal float32 rate. One unit is one head; per GPU fixed ("weak")."""

    name = "attention"
    unit = "heads/s"
    dtype = "f32"
    seq, width = 8192, 64

    def __init__(self, rank: int):
        self.rank = rank

    def config(self):
        return {"workload": f"streaming attention, one head: q, k, v [{self.seq},{self.width}] fp32 ~N(0,1); "
                            "softmax(q k^T / sqrt(64)) v in one pass over the keys",
                "flops_per_head": 4 * self.seq * self.seq * self.width, "l2": L2_NOTE}

    def setup(self, device):
        import torch

        g = torch.Generator().manual_seed(self.rank)
        self.host = [torch.randn(self.seq, self.width, generator=g).pin_memory() for _ in range(3)]
        self.dev = [t.to(device) for t in self.host]
        self.out = torch.empty_like(self.dev[0])
        self.staging = [torch.empty_like(t) for t in self.dev]
        self.out_host = torch.empty(self.seq, self.width).pin_memory()

    def launches_per_step(self) -> int:
        return 1

    def step_profiled(self) -> list[float]:
        import torch

        from tgcb import attention

        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        attention.streaming_attention_into(*self.dev, self.out)
        e.record()
        e.synchronize()
        return [s.elapsed_time(e)]

    def step_e2e(self) -> None:
        from tgcb import attention

        for d, h in zip(self.staging, self.host, strict=True):
            d.copy_(h, non_blocking=True)
        attention.streaming_attention_into(*self.staging, self.out)
        self.out_host.copy_(self.out, non_blocking=True)

    def h2d_bytes(self) -> int:
        return 3 * self.seq * self.width * 4

    def d2h_bytes(self) -> int:
        return self.seq * self.width * 4

    def kernel_work(self) -> list[dict]:
        return [{"name": "streaming_attention<64>", "kind": "attention", "bound": "fp32", "work": 4 * self.seq * self.seq * self.width}]

    @property
    def cpu_feeds(self):
        return {}

    def cpu_program(self):
        """tgc's streaming_attention restated by the oracle (torch CPU, float32, blocks of 128)."""
        import torch

        from oracle import analysis

        g = torch.Generator().manual_seed(self.rank)
        q, k, v = (torch.randn(self.seq, self.width, generator=g) for _ in range(3))
        return lambda _feeds: analysis.streaming_attention(q, k, v)


WORKLOADS = {"mlp": MlpWorkload, "cone": ConeWorkload, "int8": Int8Workload, "longsum": LongSumWorkload,
             "train": TrainWorkload, "attention": AttentionWorkload}
# timed after the headline workload in the same run, each reported under "workloads"
SUB_WORKLOADS = ("cone", "longsum", "int8", "train", "attention")


# ----------------------------------------------------------------------------- cpu baseline


def cpu_baseline(wl, budget_s: float) -> dict:
    """The oracle's restatement of tgc's CPU path, timed on the host cores."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    prog = wl.cpu_program()
    feeds = wl.cpu_feeds
    prog(feeds)
    times = []
    start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        prog(feeds)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start > budget_s or len(times) >= 50:
            break
    med = statistics.median(times) * getattr(wl, "cpu_scale", 1)
    what = (
        "oracle/bracketing.c's restatement of tgc's summation.pairwise (1 thread)"
        if wl.name == "longsum"
        else "oracle/interp.py (tgc's generated-Python executor restated: one torch CPU op per node into one arena)"
    )
    return {
        "value": 1.0 / med,
        "unit": wl.unit,
        "cores": 1 if wl.name == "longsum" else torch.get_num_threads(),
        "kind": "port",
        "sample": f"{len(times)} executions by {what}; median {med:.4f} s per unit"
        + (f" (one 8192-row shard timed, x{wl.cpu_scale} for the 65536-row step)" if getattr(wl, "cpu_scale", 1) > 1 else ""),
    }


# ----------------------------------------------------------------------------- main


def read_traffic(workload: str, kernel: str):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summary.

    Lines read ``workload kernel-name bytes  # note``; a kernel name may hold spaces. A dominant
    "kernel" named ``a+b`` (a launch and the dependent launch that finishes it) gets the sum of
    its parts when every part is listed, else None."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    if not os.path.exists(path):
        return None
    table = {}
    with open(path) as f:
        for line in f:
            if line.startswith("#"):
                continue
            parts = line.split("#", 1)[0].split()
            if len(parts) >= 3 and parts[-1].isdigit():
                table[(parts[0], " ".join(parts[1:-1]))] = int(parts[-1])
    names = kernel.split("+")
    if all((workload, n) in table for n in names):
        return sum(table[(workload, n)] for n in names)
    return None


def main() -> int:
    # The JSON line must be the only thing on stdout; libraries (NCCL prints its version on
    # rank 0) write to file descriptor 1, so point it at stderr and keep a private copy.
    sys.stdout.flush()
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr
    try:
        return _main(json_out)
    finally:
        json_out.flush()


class Runner:
    """What every workload's measurement shares: device, process group, L2 flush, timing."""

    def __init__(self, args, device, dist, n: int, rank: int, local: int):
        import torch

        self.args, self.device, self.dist, self.n, self.rank, self.local = args, device, dist, n, rank, local
        self.flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.flush_read = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.flush_sink = torch.empty((), dtype=torch.float32, device=device)
        self.peaks, self.peak_source = peaks()

    def flush_l2(self) -> None:
        import torch

        self.flush.zero_()
        torch.sum(self.flush_read, dim=0, out=self.flush_sink)

    def timed(self, fn, steps: int) -> list[float]:
        """``steps`` calls of ``fn`` (which returns ms per launch), each after an L2 flush and a
        bounded delay kernel; returns the per-launch ms summed over the steps."""
        from tgcb.runtime import delay

        total = None
        for _ in range(steps):
            self.flush_l2()
            delay(50_000)
            ms = fn()
            total = ms if total is None else [a + b for a, b in zip(total, ms, strict=True)]
        return total

    def max_over_ranks(self, value: float) -> float:
        import torch

        if not self.dist:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def barrier(self) -> None:
        import torch

        torch.cuda.synchronize()
        if self.dist:
            self.dist.barrier()
        torch.cuda.synchronize()


def make_workload(name: str, runner: Runner):
    wl = WORKLOADS[name](runner.rank)
    if name == "train":
        wl.global_rows = runner.args.train_rows
        wl.buckets = runner.args.train_buckets
        wl.side_ctas = runner.args.train_side_ctas
        wl.setup(runner.device, runner.dist, runner.n)
    elif name == "longsum":
        wl.setup(runner.device, runner.dist, runner.n)
    else:
        wl.setup(runner.device)
    return wl


def roofline_of(wl, runner: Runner, per_launch: list[float], steps: int, clocks: dict) -> tuple[dict, list[dict]]:
    pk, src = runner.peaks, runner.peak_source
    work = wl.kernel_work()
    dom = max((i for i in range(len(per_launch)) if work[i]["bound"] != "nvlink"), key=lambda i: per_launch[i])
    dk = work[dom]
    avg_ms = per_launch[dom] / steps
    if dk["bound"] == "tensor":
        factor = 0.5 if dk.get("type") == "tf32" else 2.0
        # The burst cuBLAS rate was measured at full clocks, the sustained one under the power
        # cap at lower clocks: compare against the one whose clocks this run actually had.
        sm, sm_max = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
        burst = bool(sm and sm_max and sm >= 0.95 * sm_max)
        key = "bf16_tflops" if burst else "bf16_tflops_sustained"
        peak = pk[key] * factor
        achieved = dk["work"] / (avg_ms * 1e-3) / 1e12
        unit = "TFLOP/s" if dk.get("type") == "tf32" else "TOP/s"
        peak_note = (
            f"{'tf32' if factor == 0.5 else 'int8'} dense rate taken as {factor}x the {src} "
            f"{'burst' if burst else 'sustained'} bf16 cuBLAS rate ({pk[key]} TF/s, MEASURED_PEAKS.json {key}; "
            f"{'SM clocks stayed at max during the timed region' if burst else 'SM clocks dropped during the timed region'}); "
            "B200 dense tf32:bf16:int8 = 1:2:4"
        )
    elif dk["bound"] == "fp32":
        from tgcb import cost

        peak = cost.B200_FP32_SIMT_FLOPS / 1e12
        achieved = dk["work"] / (avg_ms * 1e-3) / 1e12
        unit = "TFLOP/s"
        peak_note = ("nominal float32 CUDA-core rate (148 SMs x 128 lanes x 2 flops per FMA x 1.965 GHz); no measured "
                     "float32 peak exists in MEASURED_PEAKS.json, so this fraction is of nominal")
    else:
        peak = pk["hbm_gbs"]
        achieved = dk["work"] / (avg_ms * 1e-3) / 1e9
        unit = "GB/s"
        peak_note = f"{src} STREAM-style copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"
    roof = {
        "bound": dk["bound"],
        "kernel": dk["name"],
        "achieved": round(achieved, 2),
        "peak": round(peak, 1),
        "unit": unit,
        "frac": round(achieved / peak, 4),
        "traffic": read_traffic(wl.name, dk["name"]),
        "peak_source": peak_note,
        **({"also": dk["also"]} if dk.get("also") else {}),
    }
    return roof, work


def model_block(wl, runner: Runner, ms_per_step: float) -> dict | None:
    """tgc's roofline model (tgcb.cost) of the step on a B200 machine made from the measured
    peaks, beside the measured time: tgc's own fused-bytes estimate of the graph, and the
    same roofline over the bytes the backend's kernel steps move."""
    from tgcb import cost

    if not hasattr(wl, "compiled") or not hasattr(wl.compiled, "lowering"):
        return None
    machine = cost.b200(runner.peaks, getattr(wl, "machine_kind", "fp32"))
    tgc_est = cost.estimate(wl.compiled.graph, machine)
    plan = cost.plan_estimate(wl.compiled, machine)
    return {
        "machine": machine.as_dict(),
        "tgc_estimate_us": round(tgc_est.seconds * 1e6, 2),
        "tgc_estimate": tgc_est.as_dict(),
        "backend_bytes_estimate_us": round(plan.seconds * 1e6, 2),
        "measured_us": round(ms_per_step * 1e3, 2),
        "measured_over_backend_estimate": round(ms_per_step * 1e-3 / plan.seconds, 3) if plan.seconds else None,
    }


def measure(name: str, runner: Runner, steps: int, warmup: int, with_cpu: bool) -> dict | None:
    """Set up one workload, time it (device events, L2 flushed, max over ranks), time its
    end-to-end path, and return rank 0's result (None on the other ranks)."""
    import torch

    args, n, rank, dist = runner.args, runner.n, runner.rank, runner.dist
    wl = make_workload(name, runner)
    scaling = getattr(wl, "scaling", "weak")
    units = wl.units_per_step(n) if hasattr(wl, "units_per_step") else n

    sampler = NvmlClockSampler(runner.local)
    if not sampler.start():
        sampler = ClockSampler(runner.local)
        sampler.start()
    warm = max(warmup, 3)
    for _ in range(warm):
        wl.step_profiled()
    runner.barrier()
    sampler.mark_start()
    per_launch = runner.timed(wl.step_profiled, steps)
    torch.cuda.synchronize()
    sampler.mark_end()
    clocks = sampler.stop()
    if hasattr(wl, "compiled"):
        wl.compiled.check_status()
    total_ms = runner.max_over_ranks(sum(per_launch))

    # end to end through the public API with host buffers
    for _ in range(2):
        wl.step_e2e()
    if hasattr(wl, "run_e2e"):
        wl.run_e2e(2)
    runner.barrier()
    e2e_ms = 0.0
    stream = torch.cuda.current_stream()
    if hasattr(wl, "run_e2e"):
        e2e_ms = wl.run_e2e(steps)
    else:
        for _ in range(steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            wl.step_e2e()
            e.record(stream)
            e.synchronize()
            e2e_ms += s.elapsed_time(e)
    e2e_ms = runner.max_over_ranks(e2e_ms)
    runner.barrier()
    extras = wl.extras(runner, steps) if hasattr(wl, "extras") else {}

    result = None
    if rank == 0:
        roof, work = roofline_of(wl, runner, per_launch, steps, clocks)
        shares = [p / sum(per_launch) for p in per_launch]
        value = units * steps / (total_ms * 1e-3)
        hbm_bytes = sum(w["work"] for w in work if w["bound"] == "hbm")
        hbm_ms = sum(per_launch[i] for i, w in enumerate(work) if w["bound"] == "hbm") / steps
        if hasattr(wl, "parallelism"):
            parallelism = wl.parallelism(n)
        elif name == "train":
            parallelism = f"dp{n}: {wl.global_rows // n} rows per GPU" if n == 1 else f"dp{n}: {wl.global_rows // n} rows per GPU, gradients averaged " + {
                "final": "by NCCL in one grouped call after the backward",
                "per_gradient": "by NCCL per gradient, overlapped with the backward",
                "two": "by NCCL in two grouped calls: dW1 and db1 beside the last GEMM (dW2), dW2 and db2 after it",
                "peer": "by tgcb's own all-reduce over NVLink peer memory: dW1 and db1 beside the last GEMM (dW2), "
                        "dW2 and db2 after it",
            }[args.train_buckets]
        else:
            parallelism = f"dp{n}: independent row shards per GPU, no collective"
        result = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": wl.unit,
            "n_gpus": n,
            "steps": steps,
            "warmup": warm,
            "ms_per_step": round(total_ms / steps, 4),
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": wl.dtype,
            "data": "synthetic: seeded torch.randn inputs and random-init weights of the workload's shapes",
            "config": {**wl.config(), "parallelism": parallelism},
            "roofline": roof,
            "hbm_kernels": {
                "algorithmic_bytes_per_exec": hbm_bytes,
                "achieved_gbs": round(hbm_bytes / (hbm_ms * 1e-3) / 1e9, 1) if hbm_ms > 0 else None,
                "frac_of_measured_hbm": round(hbm_bytes / (hbm_ms * 1e-3) / 1e9 / runner.peaks["hbm_gbs"], 4)
                if hbm_ms > 0 else None,
            },
            "kernels": [
                {"name": w["name"], "kind": w["kind"], "avg_ms": round(per_launch[i] / steps, 4), "share": round(shares[i], 4)}
                for i, w in enumerate(work)
            ],
            "e2e": {
                "value": round(units * steps / (e2e_ms * 1e-3), 3),
                "unit": wl.unit,
                "h2d_bytes_per_step": wl.h2d_bytes(),
                "d2h_bytes_per_step": wl.d2h_bytes(),
                "how": ("compiled.function(arena, pinned host feeds, stream) then a copy of every output to pinned host "
                        "memory, calls alternating two streams and two arenas so copies overlap the neighbouring calls"
                        if hasattr(wl, "run_e2e") else "one call at a time: pinned host inputs copied in, result copied out"),
            },
            "gpu_launches": steps * wl.launches_per_step(),
            "clocks": clocks,
        }
        model = model_block(wl, runner, total_ms / steps)
        if model:
            result["model"] = model
        result.update(extras or {})
        if with_cpu:
            result["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
    if hasattr(wl, "close"):
        wl.close()  # collective where the workload shares memory with the other ranks
    del wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    runner.barrier()
    return result


def _main(json_out) -> int:
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(world, 1)

    if args.impl == "reference":
        if rank != 0:
            return 0
        return run_reference(args, n, json_out)

    if world > 1:
        # communicator set-up lines on stderr (which ranks joined, over which transport); NCCL
        # reads these once, when torch first loads it, so they are set before torch is imported
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION", "WARN"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist_mod

        dist_mod.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
        dist = dist_mod

    runner = Runner(args, device, dist, n, rank, local)
    result = measure(args.workload, runner, args.steps, args.warmup, with_cpu=(n == 1 and not args.no_cpu_baseline))
    if not args.only:
        nested = {}
        for name in SUB_WORKLOADS:
            if name == args.workload:
                continue
            nested[name] = measure(name, runner, args.sub_steps or args.steps, 3, with_cpu=False)
        if result is not None:
            result["workloads"] = nested
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), file=json_out, flush=True)
    return 0


def run_reference(args, n: int, json_out) -> int:
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    wl = WORKLOADS[args.workload](0)
    if args.workload == "longsum":
        from tgcb import workloads

        wl.v, _ = workloads.longsum_input(wl.n)
    elif args.workload == "train":
        wl.cpu_feeds = {}
    else:
        wl.g = wl.graph()
        wl.cpu_feeds = wl.feeds()
    prog = wl.cpu_program()
    feeds = wl.cpu_feeds
    warm = max(1, min(args.warmup, 2))
    for _ in range(warm):
        prog(feeds)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        prog(feeds)
        times.append(time.perf_counter() - t0)
    total = sum(times) * getattr(wl, "cpu_scale", 1)
    value = args.steps / total
    cores = 1 if args.workload == "longsum" else torch.get_num_threads()
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": wl.unit,
        "n_gpus": n,
        "steps": args.steps,
        "warmup": warm,
        "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": getattr(wl, "scaling", "weak"),
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded torch.randn inputs and random-init weights of the workload's shapes",
        "config": {**wl.config(), "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {
            "value": round(value, 4),
            "unit": wl.unit,
            "cores": cores,
            "kind": "port",
            "sample": "each step one full execution of the workload by oracle/ (tgc's CPU path restated; "
            "tgc's own source is not present on the GPU hosts)",
        },
        "e2e": {"value": round(value, 4), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), file=json_out, flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
