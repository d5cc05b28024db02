"""The timing harness on the GPU: CUDA-event timing of a libmt kernel and the
ABBA comparison of two launches of known relative cost (the same SwiGLU
kernel over n and over n/2 elements, both larger than L2): the smaller one
must resolve as a win, at close to half the time."""
import pytest
import torch

from metal_autotune_b200 import lib
from metal_autotune_b200.autotuner_runtime import measure

pytestmark = pytest.mark.gpu


def test_compare_resolves_half_the_work(cuda):
    n = 1 << 27  # 256 MB per bf16 operand: every sample streams from HBM
    g = torch.randn(n, device="cuda").to(torch.bfloat16)
    u = torch.randn(n, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(g)
    half = n // 2

    def full():
        lib.swiglu(g, u, out=out)

    def halved():
        lib.swiglu(g[:half], u[:half], out=out[:half])

    s = measure.Session()
    c = measure.compare(s, full, halved, pairs=4)
    assert c.wins_by(0.0) and not c.loses_by(0.0)
    assert 0.35 < c.median_ratio < 0.7, c.median_ratio
    assert c.well_formed()


def test_time_steps_scales_with_steps(cuda):
    x = torch.randn(1 << 26, device="cuda").to(torch.bfloat16)
    y = torch.empty_like(x)
    f = lambda: lib.swiglu(x, x, out=y)
    for _ in range(3):
        f()
    one = min(measure.time_steps(f, 10) for _ in range(3)) / 10
    many = min(measure.time_steps(f, 40) for _ in range(3)) / 40
    assert 0.7 < many / one < 1.3
