"""The reverse-mode training step on the GPU: one rank against the whole-batch oracle, and
(when two GPUs are visible) two NCCL ranks against one. TF32 GEMMs: tolerance 5e-3 of the
largest gradient entry."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import interp
from tgcb import parallel, workloads

pytestmark = pytest.mark.gpu
TF32_TOL = 5e-3


def rel_err(a, b) -> float:
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def test_single_rank_step_matches_oracle(cuda):
    rows = 512
    feeds = workloads.mlp_inputs(rows=rows, target=True)
    step = parallel.DataParallelTrainStep(rows, 1, 0)
    grads = step.step({k: v.cuda() for k, v in feeds.items()})
    torch.cuda.synchronize()
    step.compiled.check_status()
    ref = interp.run(step.graph, feeds)
    for g, r in zip(grads, ref, strict=True):
        assert rel_err(g, r) < TF32_TOL


def test_two_buckets_split_at_the_last_gemm(cuda):
    """With buckets="two" the gradients final before the last GEMM launch (dW1, db1: the last
    GEMM computes dW2) form the early bucket; dW2 and db2 the late one. On one rank the step is
    the plain step."""
    rows = 512
    feeds = workloads.mlp_inputs(rows=rows, target=True)
    step = parallel.DataParallelTrainStep(rows, 1, 0, buckets="two")
    names = list(step.compiled.module.output_names)
    assert sorted(step.early_outs + step.late_outs) == list(range(len(names)))
    assert [names[i] for i in step.early_outs] and [names[i] for i in step.late_outs]
    kinds = [s.kind for s in step.compiled.module.steps for _ in s.launches]
    assert kinds[step.early_end - 1] != "gemm" or step.early_end < len(kinds)
    assert "gemm" in kinds[step.early_end:]  # the last GEMM runs after the early bucket is final
    grads = step.step({k: v.cuda() for k, v in feeds.items()})
    torch.cuda.synchronize()
    ref = interp.run(step.graph, feeds)
    for g, r in zip(grads, ref, strict=True):
        assert rel_err(g, r) < TF32_TOL


@pytest.mark.parametrize("rows", [8192, 65536])
def test_full_size_step_matches_oracle(cuda, rows):
    """The training step at the sizes the benchmark runs: one 8192-row shard (8 GPUs) and the
    whole 65536-row batch on one GPU, d 1024, f 4096, compiled exactly as the benchmark compiles
    it (GEMM chains, row prologues and the split rules on), all four gradients against the
    oracle's whole-graph interpreter within 5e-3 of each gradient's largest entry."""
    feeds = workloads.mlp_inputs(rows=rows, target=True)
    step = parallel.DataParallelTrainStep(rows, 1, 0)
    grads = step.step({k: v.cuda() for k, v in feeds.items()})
    torch.cuda.synchronize()
    step.compiled.check_status()
    torch.set_num_threads(os.cpu_count() or 1)
    ref = interp.run(step.graph, feeds)
    for g, r in zip(grads, ref, strict=True):
        assert g.shape == r.shape
        assert rel_err(g, r) < TF32_TOL


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank: int, world: int, port: int, rows: int, out_dir: str, buckets: str = "final") -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        feeds = workloads.mlp_inputs(rows=rows, target=True)
        step = parallel.DataParallelTrainStep(rows, world, rank, dist=dist, device=dev, buckets=buckets)
        x, t = step.shard(feeds["x"], feeds["target"])
        shard = {**{k: feeds[k] for k in parallel.GRADS}, "x": x.contiguous(), "target": t.contiguous()}
        grads = step.step({k: v.to(dev) for k, v in shard.items()})
        torch.cuda.synchronize()
        torch.save([g.cpu() for g in grads], os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("buckets", ["final", "two", "per_gradient"])
def test_two_nccl_ranks_match_the_whole_batch(tmp_path, buckets):
    rows, world = 1024, 2
    mp.start_processes(_nccl_rank, args=(world, _free_port(), rows, str(tmp_path), buckets), nprocs=world, start_method="spawn")
    feeds = workloads.mlp_inputs(rows=rows, target=True)
    ref = interp.run(parallel.train_graph(rows), feeds)
    r0 = torch.load(os.path.join(tmp_path, "rank0.pt"))
    r1 = torch.load(os.path.join(tmp_path, "rank1.pt"))
    for a, b, r in zip(r0, r1, ref, strict=True):
        assert torch.equal(a, b)
        assert rel_err(a, r) < TF32_TOL


def _peer_rank(rank: int, world: int, port: int, rows: int, out_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        feeds = workloads.mlp_inputs(rows=rows, target=True)
        peer_step = parallel.DataParallelTrainStep(rows, world, rank, dist=dist, device=dev, buckets="peer")
        nccl_step = parallel.DataParallelTrainStep(rows, world, rank, dist=dist, device=dev, buckets="final")
        x, t = peer_step.shard(feeds["x"], feeds["target"])
        shard = {k: v.to(dev) for k, v in {**{k: feeds[k] for k in parallel.GRADS}, "x": x.contiguous(),
                                           "target": t.contiguous()}.items()}
        runs = []
        for _ in range(3):  # three steps: the flags' epochs advance, nothing is reset
            runs.append([g.clone() for g in peer_step.step(shard)])
        torch.cuda.synchronize()
        peer_step.compiled.check_status()
        ref = nccl_step.step(shard)
        torch.cuda.synchronize()
        torch.save({"peer": [[g.cpu() for g in r] for r in runs], "nccl": [g.cpu() for g in ref]},
                   os.path.join(out_dir, f"peer{rank}.pt"))
        peer_step.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_peer_allreduce_matches_nccl(tmp_path):
    """buckets="peer": the library's own all-reduce over NVLink peer memory. With two ranks the
    rank-order sum a + b and NCCL's are the same additions, and the average of two is exact
    scaling, so the gradients equal NCCL's bit for bit; they are the same on both ranks and
    on every step, and match the whole-batch oracle."""
    rows, world = 1024, 2
    mp.start_processes(_peer_rank, args=(world, _free_port(), rows, str(tmp_path)), nprocs=world, start_method="spawn")
    feeds = workloads.mlp_inputs(rows=rows, target=True)
    ref = interp.run(parallel.train_graph(rows), feeds)
    got = [torch.load(os.path.join(tmp_path, f"peer{r}.pt")) for r in range(world)]
    for r in range(world):
        for run in got[r]["peer"]:
            for a, b in zip(run, got[0]["peer"][0], strict=True):
                assert torch.equal(a, b)
        for a, b in zip(got[r]["peer"][0], got[r]["nccl"], strict=True):
            assert torch.equal(a, b)
    for a, r in zip(got[0]["peer"][0], ref, strict=True):
        assert rel_err(a, r) < TF32_TOL


def _nccl_sum_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch.distributed as dist

    from tgcb import summation

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        v, _ = workloads.longsum_input()
        s = summation.ShardedPairwise(v.numel(), rank, world, dist, dev)
        a, b = s.ranges[rank]
        got = s(v[a:b].to(dev))
        torch.save(torch.tensor([got], dtype=torch.float64), os.path.join(out_dir, f"sum{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_sum_the_long_vector_bit_exact(tmp_path):
    import json

    from conftest import GOLDEN

    world = 2
    mp.start_processes(_nccl_sum_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    with open(os.path.join(GOLDEN, "summation.json")) as f:
        want = json.load(f)["longsum"]["pairwise"]
    for r in range(world):
        assert float(torch.load(os.path.join(tmp_path, f"sum{r}.pt"))[0]) == want


def test_gradients_match_torch_autograd(cuda):
    """The reverse-mode graph's gradients on the GPU against torch.autograd of the same MLP loss
    in float64 on the CPU (independent of tgc's rules and of the oracle; TF32 tolerance)."""
    import math

    rows = 512
    feeds = workloads.mlp_inputs(rows=rows, target=True)
    step = parallel.DataParallelTrainStep(rows, 1, 0)
    grads = step.step({k: v.cuda() for k, v in feeds.items()})
    torch.cuda.synchronize()
    step.compiled.check_status()
    p = {k: feeds[k].double().requires_grad_(k in parallel.GRADS) for k in feeds}
    x = p["x"]
    cen = x - x.mean(1, keepdim=True)
    ln = cen / torch.sqrt((cen * cen).mean(1, keepdim=True) + workloads.LN_EPS)
    h = ln @ p["w1"] + p["b1"]
    g = 0.5 * h * (1 + torch.tanh(math.sqrt(2 / math.pi) * (h + 0.044715 * h ** 3)))
    y = g @ p["w2"] + p["b2"]
    loss = ((y - p["target"]) ** 2).mean()
    ref = torch.autograd.grad(loss, [p[k] for k in parallel.GRADS])
    for got, want in zip(grads, ref, strict=True):
        assert got.shape == want.shape
        assert rel_err(got, want) < TF32_TOL
