"""The pairwise sum split over ranks: the shard ranges are depth-k nodes of tgc's halving, and
their sums combined by a perfect tree give the whole vector's pairwise value bit for bit.

CPU only: the oracle's pairwise order (checked against tgc's values in test_oracle.py) stands
in for the kernels, and two and four gloo ranks run the exchange.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import bracketing
from tgcb import summation
from tgcb.errors import ConfigError


def perfect_tree(partials) -> np.float32:
    p = [np.float32(v) for v in partials]
    while len(p) > 1:
        p = [np.float32(p[i] + p[i + 1]) for i in range(0, len(p), 2)]
    return p[0]


def values(n: int, seed: int) -> np.ndarray:
    g = torch.Generator().manual_seed(seed)
    v = torch.rand(n, generator=g) - 0.25
    v[int(torch.randint(0, n, (1,), generator=g))] = 1e7
    return v.numpy()


@pytest.mark.parametrize("n", [64, 1000, 12345, 1000003, 1 << 20, (1 << 21) + 3])
@pytest.mark.parametrize("shards", [1, 2, 4, 8])
def test_shards_recombine_to_the_whole_sum(n, shards):
    v = values(n, n + shards)
    ranges = summation.shard_ranges(n, shards)
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    parts = [bracketing.pairwise(v[a:b]) for a, b in ranges]
    assert perfect_tree(parts) == np.float32(bracketing.pairwise(v))


@pytest.mark.parametrize("block", [1, 3, 8, 16])
def test_shards_recombine_for_every_block(block):
    n = 99991
    v = values(n, block)
    ranges = summation.shard_ranges(n, 8, block)
    assert perfect_tree([bracketing.pairwise(v[a:b], block) for a, b in ranges]) == np.float32(bracketing.pairwise(v, block))


def test_levels_and_ranges():
    assert summation.levels_for(1 << 26, 8) == 23
    assert summation.levels_for(8, 8) == 0
    assert summation.subtree_range(11, 1, 0) == (0, 5) and summation.subtree_range(11, 1, 1) == (5, 11)
    assert summation.subtree_range(11, 2, 3) == (8, 11)


def test_refusals():
    with pytest.raises(ConfigError, match="power of two"):
        summation.shard_ranges(1 << 20, 3)
    with pytest.raises(ConfigError, match="inside the tree"):
        summation.shard_ranges(40, 16)  # 40 values in blocks of 8: 40, 20, 10 split; 5 does not
    assert [b - a for a, b in summation.shard_ranges(40, 8)] == [5] * 8
    with pytest.raises(ConfigError):
        summation.subtree_range(10, 1, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


N = 300007


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        v = values(N, 7)

        def shard_sum(local, out):
            out.fill_(float(bracketing.pairwise(local.numpy())))

        def tree(partials, out):
            out.fill_(float(perfect_tree(partials.numpy())))

        s = summation.ShardedPairwise(N, rank, world, dist, "cpu", shard_sum=shard_sum, tree=tree)
        a, b = s.ranges[rank]
        with pytest.raises(ConfigError):
            s(torch.from_numpy(v[a:b - 1].copy()))
        result = s(torch.from_numpy(v[a:b].copy()))
        torch.save(torch.tensor([result], dtype=torch.float64), os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_agree_with_the_whole_sum(tmp_path, world):
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    want = float(np.float32(bracketing.pairwise(values(N, 7))))
    got = [float(torch.load(os.path.join(tmp_path, f"rank{r}.pt"))[0]) for r in range(world)]
    assert got == [want] * world
