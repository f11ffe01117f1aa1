"""The graph fuzzer's host side: tgc's generator restated (graphs print as tgc prints them),
the oracle pinned on those graphs against tgc's own interpreter, arena plans of every
generated graph, and shrinking (the planted mistake lives in the oracle side, on the CPU)."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import interp
from tgcb import fuzz, serialize
from tgcb.errors import ConfigError, VerificationError


@pytest.fixture(scope="module")
def gold():
    with open(os.path.join(GOLDEN, "fuzz.json")) as f:
        texts = json.load(f)
    return texts, np.load(os.path.join(GOLDEN, "fuzz.npz"))


def test_generator_prints_tgc_graphs(gold):
    texts, _ = gold
    for name, d in texts.items():
        cfg = fuzz.GeneratorConfig(**d["config"])
        for seed, text in enumerate(d["graphs"]):
            assert serialize.dumps(fuzz.generate(cfg, seed)) == text, (name, seed)


def test_oracle_and_feeds_pinned_on_generated_graphs(gold):
    texts, arrays = gold
    for name, d in texts.items():
        cfg = fuzz.GeneratorConfig(**d["config"])
        for seed in range(len(d["graphs"])):
            g = fuzz.generate(cfg, seed)
            feeds = fuzz.feeds_for(g, seed)
            ref_feeds = interp.random_feeds(g, seed=seed, positive=True)
            assert all(torch.equal(feeds[k], ref_feeds[k]) for k in feeds)
            for i, out in enumerate(interp.run(g, feeds)):
                assert np.array_equal(out.numpy(), arrays[f"{name}/{seed}/{i}"]), (name, seed, i)


@pytest.mark.parametrize("config", [None, fuzz.GeneratorConfig(nodes=16, inputs=3, rows=48, columns=200, reduction_chance=0.25)])
def test_every_generated_graph_gets_a_valid_plan(config):
    report = fuzz.fuzz_allocation(40, config)
    assert report.clean, [f.as_dict() for f in report.failures]


def _drop_last_binary(graph):
    """A wrong rewrite on purpose (tgc/verify/fuzz.py:300-313): the last binary node replaced
    by its left operand."""
    for index in range(len(graph.nodes) - 1, -1, -1):
        if len(graph.nodes[index].inputs) == 2:
            candidate = fuzz.drop_node(graph, index)
            if candidate is not None:
                return candidate
    return graph


def test_shrink_reduces_a_planted_failure():
    def fails(g):
        feeds = fuzz.feeds_for(g, 0)
        return not fuzz.outputs_agree(interp.run(g, feeds), interp.run(_drop_last_binary(g), feeds))

    seed = next(s for s in range(50) if fails(fuzz.generate(seed=s)))
    big = fuzz.generate(seed=seed)
    small = fuzz.shrink(big, fails)
    assert fails(small)
    assert len(small.nodes) < len(big.nodes)
    assert len(small.nodes) <= 3
    with pytest.raises(VerificationError):
        fuzz.shrink(small, lambda g: False)


def test_statistics_and_config_checks():
    stats = fuzz.generated_graph_statistics(30)
    assert stats["graphs"] == 30 and stats["reductions"] > 0 and stats["values_read_more_than_once"] > 0
    with pytest.raises(ConfigError):
        fuzz.GeneratorConfig(nodes=0)
    with pytest.raises(ConfigError):
        fuzz.GeneratorConfig(reduction_chance=2.0)
    with pytest.raises(ConfigError):
        fuzz.generate_many(0)
