"""bench.py's host-side pieces on CPU: the reference arm's JSON line (the contract the driver
parses), the row windows the in-run parity check samples, and the CPU baseline legs."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_sample_windows_cover_both_ends_and_stay_inside():
    for lo, hi in ((0, 131072), (65536, 131072), (0, 300), (10, 10), (5, 600)):
        w = bench.sample_windows(lo, hi)
        if hi <= lo:
            assert w == []
            continue
        assert w[0][0] == lo and w[-1][1] == hi
        assert all(lo <= a < b <= hi for a, b in w)


def test_dense_configs_match_baseline_shapes():
    assert bench.DENSE["5"][:4] == (1, 131072, 16, 128) and bench.DENSE["5"][7] == 0.5
    assert bench.DENSE["2"][:4] == (1, 8192, 16, 64)
    assert bench.DENSE["3"][6] == dict(softcap=30.0, window_size=(1024, 1024))
    assert bench.DENSE["1"][4] is not None and bench.DENSE["1"][5] is False


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"


def test_config1_cpu_baseline_runs_whole_problem():
    d = bench.cpu_config1_run(reps_budget_s=0.2)
    assert d["value"] > 0 and d["reps"] >= 5 and "config 1" in d["sample"]
