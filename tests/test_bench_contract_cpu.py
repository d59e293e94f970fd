"""bench.py's command-line contract where it needs no GPU: the reference arm prints exactly one JSON line
(``impl: reference`` with an ``unavailable`` reason) for workloads the reference cannot run, the warm-up
floor is enforced, and the own arm refuses to run without a CUDA device instead of timing the CPU."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def _bench(*args: str) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, capture_output=True, text=True, timeout=300)


@pytest.mark.parametrize("workload", ["qwen3-8b-cp-ring", "qwen3-32b-tp", "qwen3-vl-8b"])
def test_reference_arm_unavailable_line(workload):
    sys.path.insert(0, str(ROOT))
    from baseline.reference_arm import NOT_IN_REFERENCE

    assert workload in NOT_IN_REFERENCE
    r = _bench("--impl", "reference", "--workload", workload)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    row = json.loads(lines[0])
    assert row["impl"] == "reference" and workload in row["unavailable"]


def test_warmup_floor():
    r = _bench("--warmup", "2")
    assert r.returncode != 0 and "warmup" in r.stderr


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a CUDA device")
def test_own_arm_needs_cuda():
    r = _bench("--steps", "1", "--warmup", "3")
    assert r.returncode != 0 and "no CUDA device" in r.stderr
    ref = _bench("--impl", "reference")
    assert ref.returncode == 0 and json.loads(ref.stdout.strip().splitlines()[-1])["impl"] == "reference"
