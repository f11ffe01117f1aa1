"""Compiled-graph cache: tgc's shape signature restated (pinned to tgc's own hashes of every
golden graph), eviction policies with a counting stand-in for the compiler, and the on-disk
text index."""

from __future__ import annotations

import json
import os

import pytest
from conftest import GOLDEN

from tgcb import cache, fuzz, ir, serialize, workloads
from tgcb.errors import ConfigError


@pytest.fixture(scope="module")
def sigs():
    with open(os.path.join(GOLDEN, "signatures.json")) as f:
        return json.load(f)


def test_signatures_match_tgc(sigs):
    for name, want in sigs["graphs"].items():
        with open(os.path.join(GOLDEN, "graphs", name)) as f:
            assert cache.shape_signature(serialize.loads(f.read())) == want, name
        assert sigs["renamed"][name] == want  # tgc's own hash ignores names
    with open(os.path.join(GOLDEN, "fuzz.json")) as f:
        texts = json.load(f)
    for cfg, d in texts.items():
        for text, want in zip(d["graphs"], sigs["fuzz"][cfg], strict=True):
            assert cache.shape_signature(serialize.loads(text)) == want


def test_shapes_are_part_of_the_key():
    a = workloads.mlp_graph(ir.Builder, rows=64)
    b = workloads.mlp_graph(ir.Builder, rows=128)
    assert cache.structural_hash(a) != cache.structural_hash(b) or cache.shape_signature(a) != cache.shape_signature(b)
    assert cache.shape_signature(a) == cache.shape_signature(workloads.mlp_graph(ir.Builder, rows=64))


class Counting:
    def __init__(self):
        self.calls = 0

    def __call__(self, graph, **kw):
        self.calls += 1
        return ("compiled", cache.shape_signature(graph), self.calls)


def graphs(n):
    return [fuzz.generate(fuzz.GeneratorConfig(rows=4 + i, columns=4), seed=0) for i in range(n)]


def test_hits_return_the_same_object():
    comp = Counting()
    pc = cache.PlanCache(4, compile=comp)
    g = graphs(1)[0]
    first = pc.get(g)
    again = pc.get(fuzz.generate(fuzz.GeneratorConfig(rows=4, columns=4), seed=0))  # rebuilt, renamed nothing
    assert first is again and comp.calls == 1
    assert pc.stats.as_dict()["hits"] == 1 and pc.stats.misses == 1 and g in pc


def test_lru_thrashes_on_a_cycle_one_longer_than_the_cache():
    """tgc's documented failure mode of least-recently-used (cache.py:20-24)."""
    gs = graphs(4)
    pc = cache.PlanCache(3, "least recently used", compile=Counting())
    for _ in range(5):
        for g in gs:
            pc.get(g)
    assert pc.stats.hits == 0 and pc.stats.evictions == 17
    rnd = cache.PlanCache(3, "random", compile=Counting(), seed=1)
    for _ in range(5):
        for g in gs:
            rnd.get(g)
    assert rnd.stats.hits > 0


def test_lfu_keeps_the_common_shape():
    gs = graphs(5)
    pc = cache.PlanCache(2, "least frequently used", compile=Counting())
    for g in gs[1:]:
        pc.get(gs[0])
        pc.get(gs[0])
        pc.get(g)
    assert (cache.shape_signature(gs[0]), None) in pc.keys()
    fifo = cache.PlanCache(2, "first in", compile=Counting())
    for g in gs[:3]:
        fifo.get(g)
    assert [k[0] for k in fifo.keys()] == [cache.shape_signature(g) for g in gs[1:3]]


def test_directory_index_and_warm(tmp_path):
    gs = graphs(3)
    pc = cache.PlanCache(8, directory=str(tmp_path), compile=Counting())
    for g in gs:
        pc.get(g)
    files = sorted(os.listdir(tmp_path))
    assert len(files) == 3 and all(f.endswith(".tgc") for f in files)
    fresh = cache.PlanCache(8, directory=str(tmp_path), compile=Counting())
    assert fresh.warm() == 3
    assert all(g in fresh for g in gs)
    for g in gs:
        fresh.get(g)
    assert fresh.stats.hits == 3


def test_refusals():
    with pytest.raises(ConfigError):
        cache.PlanCache(0)
    with pytest.raises(ConfigError):
        cache.PlanCache(2, "optimal")
