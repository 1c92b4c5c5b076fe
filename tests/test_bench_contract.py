"""bench.py's reference arm on the host (no GPU): the JSON line the driver reads, and the
torchrun rule that ranks other than 0 print nothing and exit 0.  The arm times the
reference's own CPU matvec / matmul (oracle/_ref when it was built here, else the
oracle's restatement) on bounded samples, so each run takes a few seconds."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           *args], cwd=ROOT, env=env, capture_output=True, text=True, timeout=240)


@pytest.mark.parametrize("workload,unit", [("matvec-i4", "GB/s"), ("matmul-i4", "TFLOP/s")])
def test_reference_arm_line(workload, unit):
    r = _run(["--workload", workload, "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d)
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0
    assert d["higher_is_better"] is True
    assert d["config"]["workload"].startswith(workload)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_silent():
    r = _run(["--workload", "matvec-i4", "--steps", "1", "--warmup", "3"],
             {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
