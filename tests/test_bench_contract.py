"""bench.py prints one JSON line with the keys its consumers read: the CPU reference arm (the C
oracle on a bounded sample) here, and the GPU arm on a one-layer case of the 7B model."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, timeout):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, capture_output=True,
                       text=True, timeout=timeout)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"], 600)
    assert d["impl"] == "reference"
    for k in ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "dtype", "data", "config"]:
        assert k in d, k
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["value"] > 0 and d["higher_is_better"] is True


@pytest.mark.gpu
def test_gpu_arm_line():
    d = _run(["--layers", "1", "--steps", "3", "--warmup", "3", "--no-e2e", "--no-one-at-a-time", "--no-micro",
              "--no-cpu-baseline", "--no-strong"], 900)
    for k in ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "roofline", "clocks", "e2e", "gpu_launches"]:
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3 and d["scaling"] == "weak"
    assert d["value"] > 0 and d["gpu_launches"] > 0 and "workload" in d["config"]
    r = d["roofline"]
    for k in ["bound", "achieved", "peak", "unit", "frac", "traffic"]:
        assert k in r, k
    assert r["bound"] == "hbm" and 0 < r["frac"] == pytest.approx(r["achieved"] / r["peak"], abs=1e-3)
    c = d["clocks"]
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(c)
    assert 0.6 < d["ratio"] < 0.7
