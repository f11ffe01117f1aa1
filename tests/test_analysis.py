"""The oracle's restatements of tgc's attention and normalisation analyses, pinned bit for
bit against outputs of tgc itself; the normalisation graphs' structure (one fused row kernel)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import analysis as oa
from tgcb import normalisation, runtime
from tgcb.attention import AttentionShape
from tgcb.errors import ConfigError

HEADS = [(256, 64, 128, 0, 1.0), (300, 32, 50, 1, 1.0), (192, 128, 64, 2, 1.0), (200, 16, 7, 3, 8.0)]
ROWS = [(48, 512, 0.5, 0), (37, 300, 0.0, 1)]


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(GOLDEN, "analysis.npz"))


def test_attention_restatement_bit_exact(gold):
    for s, w, blk, seed, scale in HEADS:
        q, k, v = oa.random_head(s, w, seed=seed, scale=scale)
        tag = f"attn/{s}_{w}_{blk}_{seed}_{scale}"
        assert np.array_equal(oa.streaming_attention(q, k, v, blk).numpy(), gold[f"{tag}/streaming"])
        assert np.array_equal(oa.naive_attention(q, k, v).numpy(), gold[f"{tag}/naive"])


def test_normalisation_restatement_bit_exact(gold):
    for rows, width, offset, seed in ROWS:
        x, _, _ = oa.random_rows(rows, width, seed=seed, offset=offset)
        tag = f"norm/{rows}_{width}_{offset}_{seed}"
        gain, shift = torch.from_numpy(gold[f"{tag}/gain"]), torch.from_numpy(gold[f"{tag}/shift"])
        mean, var = torch.from_numpy(gold[f"{tag}/mean"]), torch.from_numpy(gold[f"{tag}/var"])
        assert np.array_equal(oa.layer_norm(x, gain, shift).numpy(), gold[f"{tag}/layer"])
        assert np.array_equal(oa.rms_norm(x, gain).numpy(), gold[f"{tag}/rms"])
        assert np.array_equal(oa.batch_norm(x, gain, shift).numpy(), gold[f"{tag}/batch"])
        assert np.array_equal(oa.batch_norm(x, gain, shift, running=(mean, var)).numpy(), gold[f"{tag}/batch_running"])


def test_row_normalisations_are_one_kernel():
    for g in (normalisation.layer_norm_graph(4096, 1024), normalisation.rms_norm_graph(4096, 1024)):
        mod = runtime.generate(g)[3]
        assert [s.kind for s in mod.steps] == ["row"]
    assert [s.kind for s in runtime.generate(normalisation.batch_norm_graph(64, 32, running=True))[3].steps] == ["map"]


def test_shapes_and_checks():
    assert AttentionShape(4096, 64).arithmetic == 4.0 * 4096 * 4096 * 64
    with pytest.raises(ConfigError):
        AttentionShape(0, 4)
    with pytest.raises(ConfigError, match="matrix"):
        normalisation.rms_norm(torch.ones(3), torch.ones(3))
    with pytest.raises(ConfigError, match="epsilon"):
        normalisation.rms_norm(torch.ones(3, 3), torch.ones(3), epsilon=0.0)
