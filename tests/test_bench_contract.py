"""CPU checks of bench.py's reference arm (the reference's FP32 CPU decode,
timed on the host cores): under a multi-rank launch only rank 0 works and
prints, and its single JSON line carries the keys the benchmark contract
asks for."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(args, **env):
    full_env = dict(os.environ, **env)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=full_env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_other_ranks_exit_without_work():
    result = _run(["--impl", "reference", "--gpus", "2"], RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    assert result.returncode == 0, result.stderr[-2000:]
    assert result.stdout.strip() == ""


def test_reference_arm_prints_one_contract_line():
    result = _run(["--impl", "reference", "--context", "64", "--steps", "1", "--warmup", "1"],
                  RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    assert result.returncode == 0, result.stderr[-2000:]
    lines = [line for line in result.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["unit"] == "ms/token" and line["higher_is_better"] is False
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 1
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "ms/token", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
