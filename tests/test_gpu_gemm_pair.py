"""The tcgen05 GEMM on CTA pairs (cta_group::2, 256 x 256 tiles) against the
single-SM form (128 x 256 tiles) and an fp32 torch product: linear with and
without bias / GELU, the residual form, the implicit-GEMM conv1d (3 taps,
stride 2) and the SwiGLU epilogue of the many-rows quantized matmul, at sizes
with partial row and column tiles. MT_GEMM_PAIR=1 / 0 selects the form.
Tolerance against fp32: one element-type ulp of the value per rounding plus
2^-8 of the largest magnitude."""
from __future__ import annotations

import pytest
import torch

from metal_autotune_b200 import lib, workload

pytestmark = pytest.mark.gpu


def _both(fn, monkeypatch):
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("MT_GEMM_PAIR", mode)
        out[mode] = fn().clone()
    monkeypatch.delenv("MT_GEMM_PAIR")
    torch.cuda.synchronize()
    return out["0"], out["1"]


def _close(got, want, dtype, roundings=2):
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    g, w = got.float(), want.float()
    tol = roundings * ulp * w.abs() + 2.0 ** -8 * w.abs().max()
    bad = (g - w).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} of {w.numel()} elements off (max diff {(g - w).abs().max():.3g})"


def _rand(*shape, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).cuda()


LINEAR = [  # M, N, K, bias, act, dtype
    (1000, 768, 512, False, 0, torch.bfloat16),   # last pair tile half live (rows 768..999)
    (300, 520, 320, True, 1, torch.float16),      # columns past 512 in a partial tile, GELU
    (2048, 1024, 64, True, 0, torch.bfloat16),    # one K-block per tile
    (4096, 2048, 1024, False, 0, torch.float16),  # many tiles per pair
]


@pytest.mark.parametrize("M,N,K,bias,act,dtype", LINEAR)
def test_linear_pairs_match_single_sm(cuda, monkeypatch, M, N, K, bias, act, dtype):
    x = _rand(M, K, dtype=dtype, seed=M)
    w = _rand(N, K, dtype=dtype, seed=N, scale=K ** -0.5)
    b = _rand(N, dtype=dtype, seed=K, scale=0.1) if bias else None
    single, pair = _both(lambda: lib.linear(x, w, b, act=act), monkeypatch)
    ref = x.float() @ w.float().t()
    if bias:
        ref = ref + b.float()
    if act:
        ref = torch.nn.functional.gelu(ref)
    _close(pair, ref, dtype, roundings=3)
    _close(pair, single, dtype)


def test_linear_residual_pairs(cuda, monkeypatch):
    M, N, K, dtype = 513, 256, 1024, torch.bfloat16
    h = _rand(M, K, dtype=dtype, seed=1)
    w = _rand(N, K, dtype=dtype, seed=2, scale=K ** -0.5)
    b = _rand(N, dtype=dtype, seed=3, scale=0.1)
    r = _rand(M, N, dtype=dtype, seed=4)
    single, pair = _both(lambda: lib.linear_residual(h, w, b, r), monkeypatch)
    _close(pair, h.float() @ w.float().t() + b.float() + r.float(), dtype, roundings=3)
    _close(pair, single, dtype)


def test_conv1d_pairs(cuda, monkeypatch):
    """Implicit-GEMM conv: 3 taps, stride 2, padding 1, two clips, bias + GELU."""
    N, L, Cin, Cout, dtype = 2, 600, 128, 384, torch.float16
    x = _rand(N, L, Cin, dtype=dtype, seed=5)
    w = _rand(Cout, 3, Cin, dtype=dtype, seed=6, scale=(3 * Cin) ** -0.5)
    b = _rand(Cout, dtype=dtype, seed=7, scale=0.1)
    single, pair = _both(lambda: lib.conv1d(x, w, b, stride=2, padding=1, act=1), monkeypatch)
    ref = torch.nn.functional.conv1d(x.float().transpose(1, 2), w.float().transpose(1, 2), b.float(), stride=2,
                                     padding=1)
    ref = torch.nn.functional.gelu(ref).transpose(1, 2)
    _close(pair, ref, dtype, roundings=3)
    _close(pair, single, dtype)


def test_swiglu_epilogue_pairs(cuda, monkeypatch):
    """Gate rows in the even CTA's weight half, up rows in the odd one's: the
    SwiGLU epilogue of the many-rows quantized matmul on pairs."""
    M, N, K, bits, dtype = 1100, 320, 512, 4, torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(8)
    wg = workload.random_quantized(N, K, bits=bits, dtype=dtype, generator=g)
    wu = workload.random_quantized(N, K, bits=bits, dtype=dtype, generator=g)
    x = _rand(M, K, dtype=dtype, seed=9)
    single, pair = _both(lambda: lib.quantized_matmul_swiglu(x, *wg, *wu, bits=bits), monkeypatch)
    gate = (x.float() @ workload.dequantize(*wg, 64, bits).float().t()).to(dtype).float()
    up = (x.float() @ workload.dequantize(*wu, 64, bits).float().t()).to(dtype).float()
    ref = torch.nn.functional.silu(gate) * up
    _close(pair, ref, dtype, roundings=4)
    _close(pair, single, dtype)


def test_pairs_are_bitwise_the_single_sm_result(cuda, monkeypatch):
    """Same K order (64-wide blocks, 16-wide MMA steps), same epilogue: the two
    forms are expected to agree bit for bit."""
    M, N, K, dtype = 1536, 1280, 2048, torch.bfloat16
    x = _rand(M, K, dtype=dtype, seed=10)
    w = _rand(N, K, dtype=dtype, seed=11, scale=K ** -0.5)
    single, pair = _both(lambda: lib.linear(x, w, None, act=0), monkeypatch)
    assert torch.equal(single, pair), int((single != pair).sum())
