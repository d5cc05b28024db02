"""Decode cuts with the RMSNorm fused into the streamed matmul's staging of x
(mt_rms_norm_quantized_matmul_multi / _swiglu): bit-identical to mt_rms_norm
followed by the unfused matmul (same sum-of-squares order, same roundings),
and within the matmul tolerance of the oracle's composition
rms_norm -> quantized_matmul (-> swiglu)."""
import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

pytestmark = pytest.mark.gpu

EPS = 1e-6


def t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype).cuda()


def n(x):
    return x.float().cpu().numpy()


def close(got, ref, *, ulps, abs_frac):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    tol = ulps * 2 ** -7 * np.abs(ref) + abs_frac * max(np.abs(ref).max(), 1e-30)
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {np.abs(got - ref).max():.4g}"


def quantized(oracle, N, K, dtype, seed):
    r = np.random.default_rng(seed)
    wq, s, b = oracle.quantize_affine(r.standard_normal((N, K)).astype(np.float32) * 0.02, 64, 4, dtype)
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    return (wq, s, b), (torch.from_numpy(wq.view(np.int32)).cuda(), t(s, tdt), t(b, tdt))


def inputs(oracle, M, K, dtype, seed):
    r = np.random.default_rng(seed)
    x = oracle.round_to(r.standard_normal((M, K)).astype(np.float32) * 3.0, dtype)
    w = oracle.round_to(1.0 + 0.25 * r.standard_normal(K).astype(np.float32), dtype)
    return x, w


MULTI_CASES = [
    # M, K, N per set, dtype
    (1, 2560, (4096, 1024, 1024), "bfloat16"),  # Qwen3-4B q/k/v at decode
    (2, 2560, (4096, 1024, 1024), "bfloat16"),
    (3, 512, (512, 256, 256), "float16"),
    (4, 1024, (300, 128), "bfloat16"),
    (1, 2560, (151936,), "bfloat16"),  # tied lm_head: scales streamed with the weight stages
]


@pytest.mark.parametrize("M,K,Ns,dtype", MULTI_CASES)
def test_norm_multi(cuda, oracle, M, K, Ns, dtype):
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    x, w = inputs(oracle, M, K, dtype, seed=M * 7 + K)
    sets = [quantized(oracle, N, K, dtype, seed=20 + i) for i, N in enumerate(Ns)]
    xt, wt = t(x, tdt), t(w, tdt)
    fused = lib.rms_norm_quantized_matmul_multi(xt, wt, EPS, [g for _, g in sets])
    xn = lib.rms_norm(xt, wt, EPS)
    plain = lib.quantized_matmul_multi(xn, [g for _, g in sets])
    torch.cuda.synchronize()
    for f, p in zip(fused, plain):
        assert torch.equal(f, p)
    if max(Ns) <= 4096:
        xr = oracle.rms_norm(x, w, EPS, dtype)
        for ((wq, s, b), _), f in zip(sets, fused):
            close(n(f), oracle.quantized_matmul(xr, wq, s, b, 64, 4, dtype), ulps=2 if dtype == "bfloat16" else 8,
                  abs_frac=2 ** -8)


@pytest.mark.parametrize("M,K,N,dtype", [(1, 2560, 9728, "bfloat16"), (4, 512, 1024, "bfloat16"),
                                         (2, 1024, 384, "float16")])
def test_norm_swiglu(cuda, oracle, M, K, N, dtype):
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    x, w = inputs(oracle, M, K, dtype, seed=M * 11 + N)
    (wg, sg, bg), gt = quantized(oracle, N, K, dtype, seed=1)
    (wu, su, bu), ut = quantized(oracle, N, K, dtype, seed=2)
    xt, wt = t(x, tdt), t(w, tdt)
    fused = lib.rms_norm_quantized_matmul_swiglu(xt, wt, EPS, *gt, *ut)
    plain = lib.quantized_matmul_swiglu(lib.rms_norm(xt, wt, EPS), *gt, *ut)
    torch.cuda.synchronize()
    assert torch.equal(fused, plain)
    xr = oracle.rms_norm(x, w, EPS, dtype)
    ref = oracle.swiglu(oracle.quantized_matmul(xr, wg, sg, bg, 64, 4, dtype),
                        oracle.quantized_matmul(xr, wu, su, bu, 64, 4, dtype), dtype)
    close(n(fused), ref, ulps=3 if dtype == "bfloat16" else 8, abs_frac=2 ** -8)


def test_norm_zero_row_and_repeat(cuda, oracle):
    """An all-zero row normalises to zeros (scale = 1/sqrt(eps)); two calls agree bitwise."""
    x, w = inputs(oracle, 2, 1024, "bfloat16", seed=3)
    x[1] = 0.0
    sets = [quantized(oracle, 256, 1024, "bfloat16", seed=5)]
    xt, wt = t(x, torch.bfloat16), t(w, torch.bfloat16)
    a = lib.rms_norm_quantized_matmul_multi(xt, wt, EPS, [g for _, g in sets])[0]
    b = lib.rms_norm_quantized_matmul_multi(xt, wt, EPS, [g for _, g in sets])[0]
    plain = lib.quantized_matmul_multi(lib.rms_norm(xt, wt, EPS), [g for _, g in sets])[0]
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, plain)


@pytest.mark.parametrize("M,K", [(5, 1024), (1, 256)])
def test_norm_outside_decode_kernel_is_refused(cuda, oracle, M, K):
    """More than 4 rows, or rows whose scale groups are below one 16-byte copy,
    are not the streamed kernel's: the call reports it and writes nothing."""
    x, w = inputs(oracle, M, K, "bfloat16", seed=9)
    sets = [quantized(oracle, 128, K, "bfloat16", seed=6)]
    xt, wt = t(x, torch.bfloat16), t(w, torch.bfloat16)
    out = torch.full((M, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(lib.MTError, match="streamed decode kernel"):
        lib.rms_norm_quantized_matmul_multi(xt, wt, EPS, [g for _, g in sets], outs=[out])
    assert bool((out == 7.0).all())
