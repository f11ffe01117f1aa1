"""The compiled-graph cache with the real compiler: a hit hands back the loaded plan, and the
plan it hands back still computes the graph (softmax fixture against the oracle, rtol 1e-5)."""

from __future__ import annotations

import os

import pytest
import torch
from conftest import GOLDEN

from oracle import interp
from tgcb import cache, serialize

pytestmark = pytest.mark.gpu


def test_plan_cache_hits_and_runs(cuda, tmp_path):
    with open(os.path.join(GOLDEN, "graphs", "fixture_softmax_graph.tgc")) as f:
        g = serialize.loads(f.read())
    pc = cache.PlanCache(2, directory=str(tmp_path))
    first = pc.get(g)
    second = pc.get(serialize.loads(serialize.dumps(g)))
    assert first is second and pc.stats.hits == 1 and pc.stats.misses == 1
    feeds = interp.random_feeds(g, seed=3, positive=True)
    out = second({k: v.cuda() for k, v in feeds.items()})
    torch.cuda.synchronize()
    for a, b in zip(out, interp.run(g, feeds), strict=True):
        torch.testing.assert_close(a.cpu(), b, rtol=1e-5, atol=1e-6)
    fresh = cache.PlanCache(2, directory=str(tmp_path))
    assert fresh.warm() == 1 and g in fresh
