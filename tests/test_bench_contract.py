"""bench.py's output contract, checked on the CPU: the reference arm prints exactly one JSON
line with the keys the driver reads, and the GPU arm refuses to run (no number) without a GPU."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args: str, timeout: int = 600) -> subprocess.CompletedProcess:
    env = {**os.environ, "CUDA_VISIBLE_DEVICES": os.environ.get("CUDA_VISIBLE_DEVICES", "")}
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=REPO, env=env)


def test_reference_arm_prints_one_json_line():
    p = _run("--impl", "reference", "--workload", "cone", "--steps", "2", "--warmup", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 2 and d["value"] > 0
    assert "workload" in d["config"]
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_gpu_arm_gives_no_number_without_a_gpu():
    p = _run("--steps", "1", "--warmup", "1", "--no-cpu-baseline", timeout=300)
    assert p.returncode != 0
    assert not [ln for ln in p.stdout.splitlines() if ln.strip().startswith("{")]


def test_traffic_lines_parse(tmp_path, monkeypatch):
    """profiles/ncu_traffic.txt: names may hold spaces; a composite "a+b" sums its listed parts."""
    sys.path.insert(0, REPO)
    import bench

    (tmp_path / "profiles").mkdir()
    (tmp_path / "profiles" / "ncu_traffic.txt").write_text(
        "# workload kernel bytes\n"
        "w void k<4> 100  # a note\n"
        "w leaf 200\n"
        "w final 5\n"
    )
    monkeypatch.setattr(bench, "REPO", str(tmp_path))
    assert bench.read_traffic("w", "void k<4>") == 100
    assert bench.read_traffic("w", "leaf+final") == 205
    assert bench.read_traffic("w", "leaf+missing") is None
    assert bench.read_traffic("other", "leaf") is None
