"""bench.py's CPU legs (the oracle on a spawn-started process pool): they run
without a GPU and report the cores they used."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_line_on_all_cores():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True,
                         timeout=300, check=True).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unit"] == "tokens/s" and rec["value"] > 0
    assert rec["cpu_baseline"]["kind"] == "port" and rec["cpu_baseline"]["cores"] >= 1
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["steps"] == 2
