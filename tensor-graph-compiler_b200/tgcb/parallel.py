"""Batch sharding across the GPUs of one box, with the gradient all-reduce done for real.

tgc simulates data parallelism in one process: ``row_parallel`` splits the batch rows over
devices with the weights replicated (tgc/parallel/shard.py:39-123), ``shard`` cuts tensors with
``torch.chunk`` and refuses a split that is not even (shard.py:57-67), and
tgc/parallel/collective.py prices the gradient all-reduce with a ring model and its overlap
with the backward pass (collective.py:76-113, 339-379). Here each rank is one process driving
one GPU; it compiles the gradient graph of its own shard (``tgcb.grad.gradient`` of the MLP's
mean-squared error over shard_rows rows, lowered by ``tgcb.runtime``), runs it, and averages
the four gradients over ranks (AVG, since every shard's loss is a mean over the same number
of rows, so the global gradient is the mean of the shard gradients). By default
(``buckets="peer"``) they are averaged by this library's own all-reduce over NVLink peer
memory (``tgcb.peer``): the step's arena is shared with the other ranks of the box, the
gradients final before the last GEMM (dW1, db1) are averaged by a kernel of ``side_ctas`` CTAs
on a side stream in the SMs that GEMM leaves free, and the rest (dW2, db2) by one CTA per SM
after it. The NCCL modes (``torch.distributed``) stay for comparison: ``"final"`` (one grouped
call after the last launch), ``"per_gradient"`` (each gradient's all-reduce on a side stream
as soon as the launch that finalises it is queued) and ``"two"`` (the peer mode's split).

The same code runs with the ``gloo`` backend on CPU ranks when ``executor`` replaces the GPU
plan (tests use the oracle there), which is how the host-side sharding and averaging logic is
tested without GPUs.
"""

from __future__ import annotations

from collections.abc import Callable

from tgcb import collective, grad, ir, workloads
from tgcb.errors import ConfigError, PassError

GRADS = ("w1", "b1", "w2", "b2")


def shard_rows(total_rows: int, devices: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of ``rank``'s contiguous block; refuses an uneven split like tgc."""
    if devices < 1:
        raise ConfigError(f"there has to be at least one device, got {devices}")
    if not 0 <= rank < devices:
        raise ConfigError(f"rank {rank} is outside {devices} devices")
    if total_rows % devices:
        raise PassError(f"{total_rows} does not divide evenly over {devices} devices")
    n = total_rows // devices
    return rank * n, n


def ring_time(size_bytes: int, devices: int, bytes_per_second: float, latency_seconds: float) -> float:
    """tgc's ring all-reduce model (collective.py:76-88) on a link of the given bandwidth and latency."""
    return collective.ring_time(size_bytes, devices, collective.Link("given", bytes_per_second, latency_seconds))


def ring_volume(size_bytes: int, devices: int) -> float:
    """Bytes each device sends in a ring all-reduce (collective.py:113-122)."""
    return collective.ring_volume(size_bytes, devices)


def train_graph(rows: int, d: int = 1024, f: int = 4096):
    """The gradient graph of mean((mlp(x) - target)^2) over ``rows`` rows w.r.t. w1, b1, w2, b2."""
    return grad.gradient(workloads.mlp_graph(ir.Builder, rows=rows, d=d, f=f, loss=True), list(GRADS), seed_is_input=False).graph


class DataParallelTrainStep:
    """One data-parallel gradient step of the MLP block (the reverse-mode workload).

    ``global_rows`` are split into ``world`` contiguous shards; rank ``rank`` owns rows
    [first, first + shard) of x and target. ``step(feeds)`` takes this rank's shard of x and
    target plus the replicated weights and returns the globally averaged gradients
    (dW1, db1, dW2, db2), identical on every rank.
    """

    def __init__(self, global_rows: int, world: int, rank: int, *, d: int = 1024, f: int = 4096, dist=None,
                 device=None, executor: Callable | None = None, buckets: str = "peer", side_ctas: int = 20):
        """``buckets``: "per_gradient" starts each gradient's all-reduce as soon as the launch that
        finalises it is queued; "final" averages all gradients in one grouped NCCL call after the
        last launch (one collective's latency instead of four; the GEMMs occupy every SM, so
        collectives queued beside them barely overlap anyway); "two" averages the gradients that
        are final before the last GEMM launch in one grouped call started on a side stream as
        soon as they are (it runs beside the last GEMM, which leaves SMs free when it has fewer
        output tiles than SM pairs), and the rest in one grouped call at the end. With NCCL the
        side call runs in its own communicator limited to ``side_ctas`` CTAs, so that it fits in
        the SMs the last GEMM leaves free instead of delaying that GEMM's resident pairs.
        "peer" splits the gradients the same way but averages them with this library's own
        all-reduce over NVLink peer memory (``tgcb.peer``; the arena is shared with the other
        ranks of the box): the early bucket in ``side_ctas`` CTAs on a side stream beside the
        last GEMM, the rest in one CTA per SM after it. Its averages are summed in rank order,
        identical on every rank and every run. The default ``side_ctas`` (20) is what the MLP's
        last GEMM (dW2: 64 pair tiles on 74 SM pairs) leaves free of the 148 SMs; on one 8-GPU
        box 20 gave 1298 steps/s and 16 gave 1277."""
        if buckets not in ("per_gradient", "final", "two", "peer"):
            raise ConfigError(f"unknown bucketing {buckets!r}")
        self.buckets = buckets
        self.global_rows = global_rows
        self.world = world
        self.rank = rank
        self.first, self.rows = shard_rows(global_rows, world, rank)
        self.dist = dist
        self.graph = train_graph(self.rows, d, f)
        self.executor = executor
        if executor is None:
            import torch

            from tgcb.runtime import compile_graph

            self.torch = torch
            self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
            self.compiled = compile_graph(self.graph, device=self.device.index)
            self.peer = None
            if buckets == "peer" and dist is not None and world > 1:
                from tgcb.peer import PeerGroup

                self.peer = PeerGroup(dist, self.compiled.arena_bytes, self.device.index)
                self.arena = self.peer.buffer
            else:
                self.arena = self.compiled.new_arena()
            self.comm = torch.cuda.Stream(device=self.device)
            # where each gradient becomes final: split the plan there
            writers = self.compiled.launch_writers()
            outs = list(self.compiled.module.output_names)
            self.finals = sorted({writers[o] for o in outs})
            self.out_at = {k: [i for i, o in enumerate(outs) if writers[o] == k] for k in self.finals}
            # "two": the launch index of the last GEMM; gradients final before it form the early bucket
            kinds = [s.kind for s in self.compiled.module.steps for _ in s.launches]
            last_gemm = max((i for i, k in enumerate(kinds) if k == "gemm"), default=len(kinds))
            early = [k for k in self.finals if k < last_gemm]
            self.early_end = (max(early) + 1) if early else 0
            self.early_outs = [i for k in early for i in self.out_at[k]]
            self.late_outs = [i for k in self.finals if k >= last_gemm for i in self.out_at[k]]
            self.side_group = None
            self.side_ctas = side_ctas
            if buckets == "two" and dist is not None and world > 1 and dist.get_backend() == "nccl":
                opts = dist.ProcessGroupNCCL.Options()
                opts.config.max_ctas = side_ctas
                self.side_group = dist.new_group(ranks=list(range(world)), backend="nccl", pg_options=opts)

    def shard(self, x, target):
        """This rank's rows of the global batch."""
        return x[self.first : self.first + self.rows], target[self.first : self.first + self.rows]

    def _average(self, tensors: list, group=None) -> None:
        if self.dist is None or self.world == 1:
            return
        if self.dist.get_backend() == "nccl":
            if len(tensors) > 1:
                from torch.distributed.distributed_c10d import _coalescing_manager

                with _coalescing_manager(group=group, device=tensors[0].device):
                    for t in tensors:
                        self.dist.all_reduce(t, op=self.dist.ReduceOp.AVG, group=group)
            else:
                self.dist.all_reduce(tensors[0], op=self.dist.ReduceOp.AVG, group=group)
        else:
            for t in tensors:
                self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
                t.div_(self.world)

    def step(self, feeds: dict, timing: list | None = None) -> list:
        """Run the step. With ``timing`` (a list), one CUDA event pair per launch is appended to
        it, recorded on the stream the launches run on."""
        if self.executor is not None:
            grads = [g.clone() for g in self.executor(self.graph, feeds)]
            self._average(grads)
            return grads
        torch = self.torch
        main = torch.cuda.current_stream(self.device)
        ptrs = self.compiled.input_pointers(self.arena, feeds)
        outs = self.compiled._outputs(self.arena, feeds)
        done = 0
        total = self.compiled.launches_per_call

        def run(first: int, count: int) -> None:
            if timing is None:
                self.compiled.run_range(self.arena, ptrs, first, count, main)
                return
            for i in range(first, first + count):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(main)
                self.compiled.run_range(self.arena, ptrs, i, 1, main)
                e.record(main)
                timing.append((s, e))

        if self.peer is not None:
            return self._peer_step(run, outs, main)
        if self.buckets == "two" and self.early_outs:
            run(0, self.early_end)
            done = self.early_end
            if self.dist is not None and self.world > 1:
                ev = torch.cuda.Event()
                ev.record(main)
                with torch.cuda.stream(self.comm):
                    self.comm.wait_event(ev)
                    self._average([outs[i] for i in self.early_outs], group=self.side_group)
        if self.buckets == "per_gradient":
            for k in self.finals:
                run(done, k + 1 - done)
                done = k + 1
                if self.dist is not None and self.world > 1:
                    ev = torch.cuda.Event()
                    ev.record(main)
                    with torch.cuda.stream(self.comm):
                        self.comm.wait_event(ev)
                        self._average([outs[i] for i in self.out_at[k]])
        if done < total:
            run(done, total - done)
        if self.buckets == "final" and self.dist is not None and self.world > 1:
            self._average(list(outs))
        if self.buckets == "two" and self.dist is not None and self.world > 1:
            self._average([outs[i] for i in (self.late_outs if self.early_outs else range(len(outs)))])
        if self.dist is not None and self.world > 1:
            main.wait_stream(self.comm)
        return outs

    def _peer_step(self, run, outs: list, main) -> list:
        from tgcb.codegen import NUM_SMS

        torch = self.torch
        total = self.compiled.launches_per_call
        done = 0
        if self.early_outs:
            run(0, self.early_end)
            done = self.early_end
            ev = torch.cuda.Event()
            ev.record(main)
            self.comm.wait_event(ev)
            self.peer.allreduce_avg([outs[i] for i in self.early_outs], 0, self.comm, self.side_ctas)
        if done < total:
            run(done, total - done)
        late = self.late_outs if self.early_outs else list(range(len(outs)))
        self.peer.allreduce_avg([outs[i] for i in late], 1, main, NUM_SMS)
        main.wait_stream(self.comm)
        return outs

    def close(self) -> None:
        """Release the peer buffers (collective: every rank calls it); the gradients returned by
        ``step`` are views of them and are invalid afterwards."""
        if getattr(self, "peer", None) is not None:
            self.peer.close()
            self.peer = None
