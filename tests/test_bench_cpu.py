"""bench.py's reference arm (the oracle on the host cores) for the star and kernel workloads: one JSON line with
the contract's keys, on the CPU (no GPU needed)."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(*args):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], capture_output=True, text=True,
                       timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("workload", ["config1", "config5a"])
def test_reference_arm_workloads(workload):
    d = run("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "0")
    assert d["impl"] == "reference" and d["unit"] == "pairs/s" and d["value"] > 0
    assert d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert workload in d["metric"]


def test_workloads_listed():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--help"], capture_output=True, text=True,
                       timeout=120, cwd=REPO)
    assert r.returncode == 0
    for w in ["config1", "config3", "config4", "config5a", "config5b-i32", "config5b-f32", "config5b-f64"]:
        assert w in r.stdout
