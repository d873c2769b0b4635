"""The benchmark's reference arm on the CPU: the JSON line it prints and its
behaviour on ranks other than 0.

`bench.py --impl reference` times the CPU restatement of the QLoRA step (the
oracle) on the host cores; it needs no GPU, so its output contract is checked
here on the smallest step workload (Qwen2.5-0.5B-shaped, one timed
iteration of the bounded sample).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(extra_env: dict[str, str]) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env.update(extra_env)
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload",
           "qwen2.5-0.5b", "--steps", "1", "--warmup", "0"]
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    out = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["steps"] == 1 and d["warmup"] == 0
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["value"] == d["value"] and cb["unit"] == "tokens/s" and cb["sample"]
    assert "workload" in d["config"]
    # The timed quantity is the sample's own wall time; the whole step it
    # stands for is reported apart from it.
    assert d["extrapolated_step_s"] * 1000.0 > d["ms_per_step"]


def test_reference_arm_is_silent_on_other_ranks():
    out = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
