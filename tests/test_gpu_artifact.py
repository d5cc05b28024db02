"""The bundle tools in a fresh process (the reference's exported
validate.py / benchmark.py, autotuner/artifact/validate.py:179-230): each is
run as `python -m metal_autotune_b200.bundles.<tool> <bundle>` in a new
interpreter that imports nothing from this test, rebuilds the seeded target
twice (original and bundle-applied), checks bitwise repeatability of both and
the patched outputs against the original's under the bundle's recorded
tolerance, and (benchmark) times both in alternated whole sequences."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
BUNDLES = ROOT / "metal_autotune_b200" / "bundles"


def _run(tool, bundle, tmp_path, *extra):
    out = tmp_path / f"{tool}_{bundle}.json"
    p = subprocess.run([sys.executable, "-m", f"metal_autotune_b200.bundles.{tool}", str(BUNDLES / bundle),
                        "--json", str(out), *extra], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.exists(), p.stderr[-2000:]
    return p.returncode, json.loads(out.read_text())


@pytest.mark.parametrize("bundle", ["tiny_mlp", "qwen3_tiny", "whisper_tiny", "mamba_tiny"])
def test_validate_in_fresh_process(cuda, bundle, tmp_path):
    rc, res = _run("validate", bundle, tmp_path)
    assert rc == 0, res
    assert res["validate"] and all(c["passed"] for c in res["validate"])
    assert all(c["cosine"] > 0.999 for c in res["validate"])


def test_benchmark_in_fresh_process(cuda, tmp_path):
    rc, res = _run("benchmark", "qwen3_tiny", tmp_path, "--steps", "3")
    assert rc == 0, res
    (row,) = res["benchmark"]
    assert row["pairs"] == 4 and row["speedup"] > 0
