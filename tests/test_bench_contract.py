"""bench.py's reference arm (the oracle port timed on the host cores) prints
the one-line JSON the driver reads: the base contract's keys plus
cpu_baseline and an e2e object with zero host<->device bytes.  Runs on CPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline",
             "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def test_reference_arm_gemv_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "gemv", "--steps", "4",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["config"]["workload"] == "config1_gemv"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
