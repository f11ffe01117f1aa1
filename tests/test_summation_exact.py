"""tgcb.summation.exact, the float64 reference the bench reports errors against, is tgc's
summation.exact (math.fsum over float64, tgc/analysis/summation.py:47-53): equal to tgc's
golden values, including the 2^26-value long sum, and to math.fsum on random magnitudes,
subnormals and cancellation."""

from __future__ import annotations

import json
import math
import os

import numpy as np
import pytest
from conftest import GOLDEN

from tgcb import summation, workloads
from tgcb.errors import ConfigError


def test_exact_matches_tgcs_golden_values():
    with open(os.path.join(GOLDEN, "summation.json")) as f:
        gold = json.load(f)
    v, _ = workloads.longsum_input()
    assert summation.exact(v) == gold["longsum"]["exact"]
    assert summation.exact(np.array([0.1, 0.2, 0.3], dtype=np.float32)) == gold["known"]["exact_0.1_0.2_0.3"]


def test_exact_matches_fsum_on_hard_inputs():
    rng = np.random.default_rng(7)
    for _ in range(100):
        a = (rng.standard_normal(500) * np.exp(rng.uniform(-100, 87, 500))).astype(np.float32)
        a[rng.integers(0, 500, 10)] = np.float32(1e-45)  # subnormals
        assert summation.exact(a) == math.fsum(a.astype(np.float64).tolist())
    big = np.array([3e38, 3e38, -3e38, 1.0], dtype=np.float32)  # the float32 sum would overflow
    assert summation.exact(big) == math.fsum(big.astype(np.float64).tolist())
    assert math.isinf(summation.exact(np.array([np.inf, 1.0], dtype=np.float32)))


def test_exact_refuses_what_tgc_refuses():
    with pytest.raises(ConfigError):
        summation.exact(np.array([], dtype=np.float32))
    with pytest.raises(ConfigError):
        summation.exact(np.array([1.0], dtype=np.float64))
    assert summation.relative_error(1.5, 1.0) == 0.5
