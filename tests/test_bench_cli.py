"""bench.py's reference arms where they cannot run: each prints one JSON line
naming why and exits 0 (the driver reads the line) -- the GPU reference arm
(the reference's own Triton kernels) on a host without CUDA, and both
reference arms for the configurations that have none."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def bench(*args: str) -> dict:
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                         text=True, cwd=ROOT, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


@pytest.mark.skipif(torch.cuda.is_available(), reason="the arm runs for real where CUDA is present")
def test_reference_gpu_arm_reports_unavailable_without_cuda():
    line = bench("--impl", "reference-gpu", "--config", "cfg2", "--steps", "3", "--warmup", "3")
    assert line["impl"] == "reference-gpu"
    assert "unavailable" in line and line["config"]["T"] == 4096


@pytest.mark.parametrize("impl", ["reference", "reference-gpu"])
@pytest.mark.parametrize("config", ["cfg2-sp", "stack"])
def test_reference_arms_unavailable_for_non_scan_configs(impl, config):
    line = bench("--impl", impl, "--config", config, "--steps", "3", "--warmup", "3")
    assert line["impl"] == impl and "unavailable" in line
