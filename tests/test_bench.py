"""bench.py's reference arm on CPU: the JSON line it prints carries the
contract's keys (metric, value, unit, cpu_baseline, e2e, config) for the
cheap workloads, timed on a short sample of the host cores."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT


@pytest.mark.parametrize("workload", ["dequant", "repack", "gemv_q6k"])
def test_reference_arm_line(workload):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--workload", workload, "--steps", "1", "--warmup", "3",
                        "--cpu-seconds", "0.3"],
                       capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    for k in ("value", "unit", "cores", "kind", "sample"):
        assert k in cb, k
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    e = d["e2e"]
    assert e["value"] == d["value"] and e["h2d_bytes_per_step"] == 0
    assert "workload" in d["config"]


def _ref_line(env_extra: dict, *args) -> dict | None:
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "20", "--warmup", "5", "--cpu-seconds", "0.3", *args],
                       capture_output=True, text=True, cwd=ROOT, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) <= 1, r.stdout
    return json.loads(lines[0]) if lines else None


def test_reference_arm_default_matches_gpu_config():
    """With no --workload, one process times the headline GEMV; its config
    carries the GPU arm's keys and values (built by the same function)."""
    import argparse

    import bench
    d = _ref_line({"WORLD_SIZE": "1", "RANK": "0"})
    rows, cols, desc = bench.WORKLOADS["gemv_up"]
    a = argparse.Namespace(workload="gemv_up", steps=20, copies=0)
    assert d["config"] == bench.gemv_config(a, 1, rows, cols, desc)
    # 20 steps over 5 copies of 33 MB: every copy waits four others before reuse
    assert d["config"]["weight_copies"] == 5


def test_reference_arm_under_torchrun_is_tp70b_on_rank0_only():
    d = _ref_line({"WORLD_SIZE": "2", "RANK": "1"})
    assert d is None
    d = _ref_line({"WORLD_SIZE": "2", "RANK": "0"})
    assert d["config"]["parallelism"] == "tp2"
    assert d["config"]["workload"].startswith("Llama-3-70B-shape")
    assert d["unit"] == "tokens/s"


def test_rotation_copies_divide_steps():
    import bench
    for steps in (1, 7, 20, 200):
        c = bench.rotation_copies(steps, 33_030_144)
        assert c * 33_030_144 >= 1.25 * bench.L2_BYTES
        assert steps % c == 0 or c > steps
