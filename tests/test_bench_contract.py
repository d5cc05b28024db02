"""The bench's JSON line contract, on the host: the reference arm (the CPU
oracle port on the host cores) prints one line with the driver's keys, its
e2e block without host<->device bytes and a cpu_baseline describing the run;
the Llama line, which has no CPU arm, prints its `unavailable` line and
exits 0. No GPU work (the reference arm never touches CUDA)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _line(*args):
    p = subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _line("--impl", "reference", "--config", "qwen3_tiny", "--steps", "1", "--warmup", "3")
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["config"]["workload"] == "qwen3_tiny"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_llama_line_has_no_cpu_arm():
    d = _line("--impl", "reference", "--config", "llama3_8b_tp")
    assert d["impl"] == "reference" and "unavailable" in d
