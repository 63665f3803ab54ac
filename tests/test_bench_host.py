"""The benchmark's host side on CPU: the reference arm's JSON line (the contract keys the
driver reads) and the sizing of the CPU baseline's row sample."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402


def test_sample_rows_whole_rows_per_thread_within_the_matrix():
    assert bench.sample_rows(15.0, 0.0041, 16) % 16 == 0
    assert bench.sample_rows(15.0, 1e-12, 16) == 16          # at least one row per thread
    assert bench.sample_rows(1e9, 1.0, 16) == bench.MM        # never more than the matrix
    # ~15 s at the measured rate: rows x 2 x 8192^2 flops / rate
    rows = bench.sample_rows(15.0, 0.004, 8)
    assert 13.0 <= rows * 2.0 * bench.MM ** 2 / 0.004e12 <= 15.0


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=300, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
