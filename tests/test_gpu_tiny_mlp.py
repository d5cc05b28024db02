"""The tiny GELU-MLP config exactly as BASELINE configs[0] defines it (seed 0,
Kaiming-uniform weights, zero biases, x ~ N(0, 1) [32, 256]) through its
bundle (try_call -> mt_linear, fp32): the first linear's pre-activation is
bit-exact against the oracle (sequential-k fused multiply-adds on both
sides); with GELU the two sides use different erf implementations (CUDA's
erff, <= 2 ulp; glibc's, <= 1 ulp), so the output agrees within the bound
derived in test_gpu_kernels.test_tiny_mlp_with_gelu_within_erf_bounds.
Bit-exactness against MLX's own CPU erf cannot be checked here (MLX is not
installed)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib
from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.targets import tiny_mlp

pytestmark = pytest.mark.gpu

BUNDLE = Path(__file__).resolve().parents[1] / "metal_autotune_b200" / "bundles" / "tiny_mlp"


def test_tiny_mlp_config_through_bundle(cuda, oracle, monkeypatch):
    monkeypatch.setenv("MT_STRICT_REGIONS", "1")
    model, x = tiny_mlp.build()
    patched = apply(model, BUNDLE)
    y = patched(x).cpu().numpy()
    xs, w1, w2 = x.cpu().numpy(), model.l1.weight.cpu().numpy(), model.l2.weight.cpu().numpy()
    b1, b2 = model.l1.bias.cpu().numpy(), model.l2.bias.cpu().numpy()
    pre = lib.linear(x, model.l1.weight, model.l1.bias, act=0).cpu().numpy()
    assert np.array_equal(pre, oracle.linear(xs, w1, b1, act=0))
    h_ref = oracle.linear(xs, w1, b1, act=1)
    ulp = np.spacing(np.abs(h_ref).astype(np.float32)).astype(np.float64)
    bound = np.abs(pre.astype(np.float64)) * 2.0 ** -22 + 4 * ulp + 1e-45
    ref = oracle.linear(h_ref, w2, b2, act=0)
    prop = np.abs(w2).sum(axis=1).max() * bound.max()
    assert np.abs(y.astype(np.float64) - ref).max() <= 4 * np.spacing(np.float32(np.abs(ref).max())) + prop
    assert patched.fallbacks == 0


def test_tiny_mlp_original_ops_agree(cuda):
    model, x = tiny_mlp.build()
    patched = apply(tiny_mlp.build()[0], BUNDLE)
    a, b = patched(x), model(x)
    assert (a - b).abs().max().item() <= 1e-5 * b.abs().max().item()
