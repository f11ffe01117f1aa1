"""CPU restatements of tgc's attention and normalisation analyses (test infrastructure only).

Same torch float32 operations in the same order as tgc/analysis/attention.py and
tgc/analysis/normalisation.py, so on the same inputs they give tgc's values bit for bit
(pinned against outputs of tgc itself in tests/golden/analysis.npz). The GPU kernels are
checked against these.
"""

from __future__ import annotations

import math

import torch


def naive_attention(queries, keys, values):
    """attention.py:81-94: the score matrix built, softmax by row maximum, then @ values."""
    scale = 1.0 / math.sqrt(queries.shape[-1])
    scores = (queries @ keys.transpose(-2, -1)) * scale
    peak = scores.amax(dim=-1, keepdim=True)
    weights = (scores - peak).exp()
    return (weights / weights.sum(dim=-1, keepdim=True)) @ values


def streaming_attention(queries, keys, values, block: int = 128):
    """attention.py:97-137: blocks of keys, running maximum and sum rescaled as they arrive."""
    scale = 1.0 / math.sqrt(queries.shape[-1])
    rows = queries.shape[0]
    running_max = torch.full((rows, 1), float("-inf"), dtype=queries.dtype)
    running_sum = torch.zeros((rows, 1), dtype=queries.dtype)
    acc = torch.zeros((rows, values.shape[-1]), dtype=queries.dtype)
    for start in range(0, keys.shape[0], block):
        kb = keys[start:start + block]
        vb = values[start:start + block]
        scores = (queries @ kb.transpose(-2, -1)) * scale
        updated = torch.maximum(running_max, scores.amax(dim=-1, keepdim=True))
        corr = (running_max - updated).exp()
        corr = torch.where(torch.isfinite(corr), corr, torch.zeros_like(corr))
        weights = (scores - updated).exp()
        running_sum = running_sum * corr + weights.sum(dim=-1, keepdim=True)
        acc = acc * corr + weights @ vb
        running_max = updated
    return acc / running_sum


def random_head(sequence: int, width: int, *, seed: int = 0, scale: float = 1.0):
    """attention.py:163-172."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sequence, width, generator=g) * scale
    k = torch.randn(sequence, width, generator=g) * scale
    v = torch.randn(sequence, width, generator=g)
    return q, k, v


def layer_norm(values, gain, offset, epsilon: float = 1e-5):
    """normalisation.py:51-58."""
    centred = values - values.mean(dim=-1, keepdim=True)
    variance = centred.pow(2).mean(dim=-1, keepdim=True)
    return centred / (variance + epsilon).sqrt() * gain + offset


def rms_norm(values, gain, epsilon: float = 1e-5):
    """normalisation.py:61-70."""
    scale = values.pow(2).mean(dim=-1, keepdim=True)
    return values / (scale + epsilon).sqrt() * gain


def batch_norm(values, gain, offset, epsilon: float = 1e-5, *, running=None):
    """normalisation.py:73-101."""
    if running is not None:
        mean, variance = running
    else:
        mean = values.mean(dim=0, keepdim=True)
        variance = values.var(dim=0, unbiased=False, keepdim=True)
    return (values - mean) / (variance + epsilon).sqrt() * gain + offset


def random_rows(rows: int, width: int, *, seed: int = 0, offset: float = 0.0):
    """normalisation.py:112-126."""
    g = torch.Generator().manual_seed(seed)
    values = torch.randn(rows, width, generator=g) + offset
    return values, torch.ones(width), torch.zeros(width)
