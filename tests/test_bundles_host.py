"""The committed region bundles are exactly what the generator writes.

`python -m metal_autotune_b200.bundles` writes every bundle under
metal_autotune_b200/bundles/ (kernels/*.launch.json, swap_table.json,
patch/wrappers.py, bundle.json); the wrapper module of each bundle is a copy
of the one committed source. Regenerating into a temporary directory must
give the committed bytes, file for file."""
from __future__ import annotations

from pathlib import Path

import pytest
import torch

from metal_autotune_b200 import bundles


def _files(d: Path) -> dict[str, bytes]:
    return {str(p.relative_to(d)): p.read_bytes() for p in sorted(d.rglob("*"))
            if p.is_file() and "__pycache__" not in p.parts}


@pytest.mark.parametrize("name,layers", [("qwen3_4b", 36), ("qwen3_tiny", 2)])
def test_committed_qwen3_bundle_is_generated(tmp_path, name, layers):
    out = bundles.write_qwen3_bundle(tmp_path / name, layers)
    assert _files(out) == _files(bundles.HERE / name)


def test_bundle_wrappers_are_the_one_source():
    src = bundles.WRAPPERS.read_bytes()
    for name in ("qwen3_4b", "qwen3_tiny"):
        assert (bundles.HERE / name / "patch" / "wrappers.py").read_bytes() == src


@pytest.mark.parametrize("name", sorted(bundles.BUNDLES))
def test_every_committed_bundle_is_generated(tmp_path, name):
    out = tmp_path / name
    bundles.BUNDLES[name](out)
    assert _files(out) == _files(bundles.HERE / name)


# ------------------------------------------------------------ fresh-process artifact tools (host side)
def test_artifact_workloads_and_builders_resolve_on_cpu():
    from metal_autotune_b200.bundles import artifact
    for name in sorted(bundles.BUNDLES):
        d = bundles.HERE / name
        meta = artifact.read_meta(d)
        assert meta["entry"] in artifact.ENTRIES
        assert meta["correctness_rule"] in ("baseline_tolerance", "exact")
        for label, w in meta["workloads"].items():
            (x,) = artifact.workload_inputs(d, w, device="cpu")
            if "seeded" in w:
                assert list(x.shape) == w["seeded"]["shape"]
                again = artifact.workload_inputs(d, w, device="cpu")[0]
                assert torch.equal(x, again)  # seeded workloads are reproducible


def test_artifact_tiny_targets_build_on_cpu():
    from metal_autotune_b200.bundles import artifact
    for name in ("qwen3_tiny", "whisper_tiny", "mamba_tiny", "tiny_mlp"):
        model = artifact.build_target(artifact.read_meta(bundles.HERE / name), device="cpu")
        assert isinstance(model, torch.nn.Module)


def test_tiny_mlp_workload_file_is_the_baseline_input():
    from metal_autotune_b200.bundles import artifact
    from metal_autotune_b200.targets import tiny_mlp
    (x,) = artifact.workload_inputs(bundles.HERE / "tiny_mlp", {"file": "workloads/x.safetensors"}, device="cpu")
    assert torch.equal(x, tiny_mlp.build(device="cpu")[1])
