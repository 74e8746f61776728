"""The reference arm of bench.py (CPU only): one JSON line with the keys the benchmark contract
asks of it, from a short run."""

import json
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    t0 = time.time()
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3", "--warmup", "3"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == "paged decode KV-read GB/s" and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True and line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert time.time() - t0 < 300


def test_warmup_below_three_is_refused():
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3", "--warmup", "2"],
                         capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert run.returncode != 0
