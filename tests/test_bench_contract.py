"""The JSON line ``bench.py --impl reference`` prints, checked on the CPU.

The reference arm times the oracle port of the reference's CPU path, so it
runs without a GPU; this pins the fields a driver reads from every bench
line (metric and unit as BASELINE.json names them, the whole-job value, the
end-to-end object with zero host traffic for a CPU run, and the CPU baseline
description).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                          cwd=REPO, capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    line = json.loads(lines[0])
    with open(os.path.join(REPO, "BASELINE.json")) as f:
        baseline = json.load(f)

    assert line["impl"] == "reference"
    assert line["metric"] == baseline["metric"]
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 1, 3)
    assert line["scaling"] in ("weak", "strong")
    assert line["data"] == "synthetic" and "workload" in line["config"]
    assert "model" not in line["config"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["kind"] in ("port", "reference")
    assert cpu["cores"] >= 1 and cpu["sample"]
