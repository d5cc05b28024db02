"""Verification fanned out one worker per GPU (metal_autotune_b200/verify.py):
three bundles checked by fresh worker processes pinned to the visible GPUs
(one at a time on a one-GPU box), each reporting one verdict."""
from pathlib import Path

import pytest
import torch

from metal_autotune_b200 import verify

pytestmark = pytest.mark.gpu

BUNDLES = Path(__file__).resolve().parents[1] / "metal_autotune_b200" / "bundles"


def test_fan_out_validates_bundles_on_every_gpu(cuda):
    names = ["tiny_mlp", "qwen3_tiny", "mamba_tiny"]
    gpus = list(range(torch.cuda.device_count()))
    vs = verify.fan_out([{"name": n, "bundle": str(BUNDLES / n)} for n in names], gpus, timeout_s=600)
    assert [v.job for v in vs] == names
    for v in vs:
        assert v.passed, v.detail
        assert v.detail["gpu"] in gpus and v.detail["checks"]


def test_ladder_jobs_climb_in_workers_one_per_gpu(cuda, monkeypatch):
    """Zoo entries as ladder jobs: each worker builds its job and climbs the
    ladder on its own GPU; the verdicts carry the gate each one stopped at."""
    import os

    import ladder_cheats as Z
    tests_dir = str(Path(__file__).resolve().parent)
    root = str(Path(__file__).resolve().parents[1])
    monkeypatch.setenv("PYTHONPATH", os.pathsep.join([tests_dir, root, os.environ.get("PYTHONPATH", "")]))
    names = ["correct", "partial_write", "eps_dropping", "atomic_racy"]
    gpus = list(range(torch.cuda.device_count()))
    vs = verify.fan_out([{"name": n, "ladder": "ladder_cheats:zoo_job", "args": [n]} for n in names], gpus,
                        timeout_s=600)
    assert [v.job for v in vs] == names
    for n, v in zip(names, vs):
        gate = Z.ZOO[n][1]
        assert v.passed == (gate is None), (n, v.detail)
        assert v.detail["failed_gate"] == gate, (n, v.detail)
        assert v.detail["gpu"] in gpus
