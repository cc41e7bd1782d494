"""bench.py's reference arm on the CPU: the JSON line the driver parses, and ranks other than 0 printing nothing.

`bench.py --impl reference` times the C restatement of the reference's CPU forward (the oracle port) on the host
cores for the headline's metric and config; it needs no GPU, so its whole contract is checked here on one series.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CMD = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
       "--cpu-series", "1"]


def run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run(CMD, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = run({"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["unit"] == "series/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1
    assert d["config"]["workload"].startswith("config5")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert "series" in cb["sample"]
    e2e = d["e2e"]
    assert e2e == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    assert run({"RANK": "1", "WORLD_SIZE": "2"}) == []
