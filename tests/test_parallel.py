"""Batch sharding and gradient averaging, as two gloo ranks on the CPU.

Each rank differentiates its own shard of the batch (the oracle stands in for the GPU plan,
so no device is needed) and the ranks average with torch.distributed; the result must equal
the gradient of the whole batch computed in one process.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import interp
from tgcb import parallel, workloads
from tgcb.errors import ConfigError, PassError

ROWS, D, F = 64, 16, 32


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        feeds = workloads.mlp_inputs(rows=ROWS, d=D, f=F, target=True)
        step = parallel.DataParallelTrainStep(ROWS, world, rank, d=D, f=F, dist=dist,
                                              executor=lambda g, fd: interp.run(g, fd))
        x, t = step.shard(feeds["x"], feeds["target"])
        shard_feeds = {**{k: feeds[k] for k in parallel.GRADS}, "x": x, "target": t}
        grads = step.step(shard_feeds)
        torch.save([g.clone() for g in grads], os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_average_to_the_full_batch_gradient(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    feeds = workloads.mlp_inputs(rows=ROWS, d=D, f=F, target=True)
    full = interp.run(parallel.train_graph(ROWS, D, F), feeds)
    r0 = torch.load(os.path.join(tmp_path, "rank0.pt"))
    r1 = torch.load(os.path.join(tmp_path, "rank1.pt"))
    for a, b, ref in zip(r0, r1, full, strict=True):
        assert torch.equal(a, b)  # every rank holds the same averaged gradient
        torch.testing.assert_close(a, ref, rtol=1e-5, atol=1e-7)


def test_shard_rows():
    assert parallel.shard_rows(65536, 8, 3) == (3 * 8192, 8192)
    with pytest.raises(PassError):
        parallel.shard_rows(10, 3, 0)
    with pytest.raises(ConfigError):
        parallel.shard_rows(10, 2, 2)


def test_ring_model():
    payload = 2 * 1024 * 4096 * 4 + 4096 * 4 + 1024 * 4  # the four MLP gradients
    assert payload == 33_574_912
    assert parallel.ring_volume(payload, 1) == 0.0
    assert parallel.ring_volume(payload, 8) == pytest.approx(2 * payload * 7 / 8)
    assert parallel.ring_time(payload, 8, 770e9, 2e-6) > parallel.ring_time(payload, 2, 770e9, 2e-6)
