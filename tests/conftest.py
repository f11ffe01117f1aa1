"""pytest configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device and the built library; everything else runs on a CPU
host. The package lives in tensor-graph-compiler_b200/ and the oracle in oracle/ at the repo
root.
"""

from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "tensor-graph-compiler_b200"))
sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and libtgcb.so")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on the CPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda:0")
