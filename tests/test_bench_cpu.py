"""bench.py's CPU legs (the reference's own PyTorch paged_decode_attention_ref
from a reference install under baseline/_ref, else the numpy oracle, on a
spawn-started process pool): they run without a GPU, sample by time and
report the cores and the kind of CPU path they used."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_line_on_all_cores():
    env = dict(os.environ, FD_REF_SECONDS="2")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True,
                         timeout=300, check=True, env=env).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["unit"] == "tokens/s" and rec["value"] > 0
    installed = (ROOT / "baseline" / "_ref" / "flashdec" / "paged_reference.py").exists()
    assert rec["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    assert rec["cpu_baseline"]["cores"] >= 1
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["steps"] == 2
    # the same config as the GPU arm (bench.c2_config), so the two lines compare
    assert rec["config"]["workload"].startswith("BASELINE c2") and rec["config"]["context"] == 2048


def test_greedy_agreement_of_the_vllm_e2e_mode():
    sys.path.insert(0, str(ROOT))
    import bench

    same = [[5, 6, 7], [1, 2, 3]]
    assert bench.greedy_agreement(same, same) == (1.0, 1.0)
    # second sequence diverges after one token, first one not at all
    first, prefix = bench.greedy_agreement(same, [[5, 6, 7], [1, 9, 3]])
    assert first == 1.0 and abs(prefix - (1.0 + 1 / 3) / 2) < 1e-12
    # a first-token flip counts against both measures
    first, prefix = bench.greedy_agreement([[4, 4]], [[3, 4]])
    assert first == 0.0 and prefix == 0.0
    # a shorter sequence only matches up to its own length
    assert bench.greedy_agreement([[1, 2, 3, 4]], [[1, 2]]) == (1.0, 0.5)
    import pytest

    with pytest.raises(ValueError):
        bench.greedy_agreement([[1]], [])
