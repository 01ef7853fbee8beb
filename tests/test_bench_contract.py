"""bench.py keeps its one-JSON-line contract: the reference arm (the
reference's CPU path, timed on the host) on any machine, and our arm on a
B200 (small case), each printing the keys a driver reads."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, timeout=600):
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, capture_output=True,
                       text=True, timeout=timeout)
    assert p.returncode == 0, f"bench.py {' '.join(args)}: exit {p.returncode}\n{p.stdout[-2000:]}\n{p.stderr[-3000:]}"
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, f"expected one JSON line, got {len(lines)}:\n{p.stdout[-2000:]}"
    return json.loads(lines[0])


def _common(j):
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "e2e"):
        assert k in j, k
    assert j["warmup"] >= 3 and j["value"] > 0 and j["higher_is_better"] is True
    assert j["unit"] == "GB/s" and j["config"]["workload"]
    for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"):
        assert k in j["e2e"], k


def test_reference_arm_line():
    j = _run("--impl", "reference", "--workload", "cfg2", "--steps", "1", "--warmup", "3")
    _common(j)
    assert j["impl"] == "reference"
    cb = j["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == j["value"] and cb["sample"]
    assert j["e2e"]["h2d_bytes_per_step"] == 0 and j["e2e"]["d2h_bytes_per_step"] == 0


@pytest.mark.gpu
def test_our_arm_line():
    j = _run("--workload", "cfg2", "--batch", "8", "--steps", "2", "--warmup", "3")
    _common(j)
    r = j["roofline"]
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] > 0 and "traffic" in r
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    assert j["gpu_launches"] > 0
    assert j["e2e"]["h2d_bytes_per_step"] > 0 and j["e2e"]["d2h_bytes_per_step"] > 0
    cb = j["cpu_baseline"]
    assert cb["cores"] >= 1 and cb["value"] > 0 and cb["kind"] in ("port", "reference")
    c = j["clocks"]
    assert "sm_mhz" in c and "sm_max_mhz" in c and "reasons" in c
    # both arms describe the same workload with the same config object
    ref = _run("--impl", "reference", "--workload", "cfg2", "--batch", "8", "--steps", "1", "--warmup", "3")
    assert ref["config"] == j["config"]
