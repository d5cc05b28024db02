"""Shared test setup. `-m gpu` tests need a CUDA device and libmt.so; the rest
run on CPU (oracle, host logic, ABI symbol checks)."""
from __future__ import annotations

import json
import math
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libmt.so")


def golden(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


def fval(v):
    """Decode the golden files' {"float": "nan"} encoding of non-finite values."""
    if isinstance(v, dict) and "float" in v:
        return float(v["float"])
    if isinstance(v, list):
        return [fval(x) for x in v]
    return v


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    from metal_autotune_b200 import build, lib
    build.build_library()
    lib.load()
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def oracle():
    from oracle import ref
    ref.lib()
    return ref
