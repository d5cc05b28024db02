"""Self-checks of the CPU oracle (no GPU): each restatement against an
independent float64 numpy evaluation of the same definition, the quantiser
round trip, and the fixed-sequence erf/exp against libm bounds."""
import math

import numpy as np
import pytest

from oracle import ref as R

rng = np.random.default_rng(0)


def bf(a):
    return R.round_to(a, "bfloat16")


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.inf, np.nan], np.float32)
    y = bf(x)
    assert y[0] == 1.0 and y[1] == 1.0 and y[2] == 1.0 + 2 ** -6 and y[3] == -2.5
    assert np.isinf(y[4]) and np.isnan(y[5])


@pytest.mark.parametrize("bits", [4, 8])
def test_quantise_round_trip(bits):
    w = rng.standard_normal((8, 128)).astype(np.float32) * 0.02
    wq, s, b = R.quantize_affine(w, 64, bits)
    q = R.unpack(wq, bits)
    assert q.max() <= (1 << bits) - 1
    deq = s.repeat(64, axis=1) * q + b.repeat(64, axis=1)
    assert np.abs(deq - w).max() <= s.max() * 0.51 + 1e-3


def _dequant64(wq, s, b, group, bits, dt="bfloat16"):
    q = R.unpack(wq, bits).astype(np.float32)
    sq = R.round_to(s.repeat(group, axis=1) * q, dt)
    return R.round_to(sq + b.repeat(group, axis=1), dt).astype(np.float64)


@pytest.mark.parametrize("bits,group", [(4, 64), (8, 64), (4, 32), (4, 128)])
def test_qmm_t_and_qmv_match_float64(bits, group):
    M, N, K = 5, 24, 256
    x = bf(rng.standard_normal((M, K)).astype(np.float32))
    wq, s, b = R.quantize_affine(rng.standard_normal((N, K)).astype(np.float32) * 0.02, group, bits)
    w = _dequant64(wq, s, b, group, bits)
    ref = x.astype(np.float64) @ w.T
    y = R.qmm_t(x, wq, s, b, group, bits)
    assert np.abs(y - ref).max() <= 2 ** -7 * np.abs(ref).max() + 1e-6
    # qmv: the affine-factored form, unrounded dequant
    q = R.unpack(wq, bits).astype(np.float64)
    ref2 = x.astype(np.float64) @ (s.repeat(group, 1).astype(np.float64) * q + b.repeat(group, 1)).T
    y2 = R.qmv(x, wq, s, b, group, bits)
    assert np.abs(y2 - ref2).max() <= 2 ** -7 * np.abs(ref2).max() + 1e-6


def test_rms_and_layer_norm_match_float64():
    x = bf(rng.standard_normal((7, 96)).astype(np.float32))
    w = bf(rng.standard_normal(96).astype(np.float32))
    y = R.rms_norm(x, w, 1e-6)
    xd = x.astype(np.float64)
    ref = xd / np.sqrt((xd ** 2).mean(-1, keepdims=True) + 1e-6) * w
    assert np.abs(y - ref).max() <= 2 ** -7 * np.abs(ref).max()
    y = R.layer_norm(x, w, w, 1e-5, "float32")
    ref = (xd - xd.mean(-1, keepdims=True)) / np.sqrt(xd.var(-1, keepdims=True) + 1e-5) * w + w
    assert np.abs(y - ref).max() < 1e-4


@pytest.mark.parametrize("traditional", [False, True])
def test_rope_matches_float64(traditional):
    H, L, D, dims, off = 3, 5, 64, 48, 7
    x = bf(rng.standard_normal((H, L, D)).astype(np.float32))
    y = R.rope(x, dims, traditional, 10000.0, 1.0, off)
    ref = x.astype(np.float64).copy()
    for l in range(L):
        for j in range(dims // 2):
            th = (l + off) * 10000.0 ** (-2 * j / dims)
            i0, i1 = (2 * j, 2 * j + 1) if traditional else (j, j + dims // 2)
            a, b = x[:, l, i0].astype(np.float64), x[:, l, i1].astype(np.float64)
            ref[:, l, i0] = a * math.cos(th) - b * math.sin(th)
            ref[:, l, i1] = a * math.sin(th) + b * math.cos(th)
    assert np.abs(y - ref).max() <= 2 ** -7 * np.abs(ref).max()
    assert np.array_equal(y[..., dims:], x[..., dims:])


@pytest.mark.parametrize("causal,off", [(True, 0), (True, 3), (False, 0)])
def test_sdpa_matches_float64(causal, off):
    B, Hq, Hkv, Lq, D = 1, 4, 2, 5, 32
    Lk = Lq + off
    q, k, v = (bf(rng.standard_normal(s).astype(np.float32)) for s in
               [(B, Hq, Lq, D), (B, Hkv, Lk, D), (B, Hkv, Lk, D)])
    o = R.sdpa(q, k, v, 0.2, causal, off)
    kk = np.repeat(k, 2, axis=1).astype(np.float64)
    vv = np.repeat(v, 2, axis=1).astype(np.float64)
    s = np.einsum("bhid,bhjd->bhij", q.astype(np.float64), kk) * 0.2
    if causal:
        s = np.where(np.arange(Lk)[None, :] <= (np.arange(Lq)[:, None] + off), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    ref = np.einsum("bhij,bhjd->bhid", p / p.sum(-1, keepdims=True), vv)
    assert np.abs(o - ref).max() <= 2 ** -7 * np.abs(ref).max() + 1e-6


def test_oracle_erf_is_the_c_library_erf():
    # the oracle's GELU uses glibc erff: within one fp32 ulp of the correctly rounded value
    for x in np.linspace(-5, 5, 2001, dtype=np.float32):
        e = math.erf(float(x))
        assert abs(R.erf(float(x)) - e) <= np.spacing(np.float32(abs(e)))


def test_swiglu_and_gelu_mlp():
    g = bf(rng.standard_normal(100).astype(np.float32))
    u = bf(rng.standard_normal(100).astype(np.float32))
    y = R.swiglu(g, u)
    ref = g / (1 + np.exp(-g.astype(np.float64))) * u
    assert np.abs(y - ref).max() < 0.02
    x = rng.standard_normal((4, 16)).astype(np.float32)
    w1, w2 = rng.standard_normal((32, 16)).astype(np.float32), rng.standard_normal((16, 32)).astype(np.float32)
    out = R.gelu_mlp(x, w1, np.zeros(32, np.float32), w2, np.zeros(16, np.float32))
    h = x.astype(np.float64) @ w1.T.astype(np.float64)
    h = 0.5 * h * (1 + np.vectorize(math.erf)(h / math.sqrt(2)))
    ref = h @ w2.T.astype(np.float64)
    assert np.abs(out - ref).max() < 1e-3


def test_logits_pick_and_embedding():
    logits = bf(rng.standard_normal(1000).astype(np.float32) * 3)
    tok, lp, lse = R.logits_pick(logits)
    assert tok == int(np.argmax(logits))
    assert abs(lse - math.log(np.exp(logits.astype(np.float64)).sum())) < 1e-4
    wq, s, b = R.quantize_affine(rng.standard_normal((50, 128)).astype(np.float32) * 0.02, 64, 4)
    out = R.quantized_embedding(np.array([3, 49, 0], np.int32), wq, s, b)
    assert np.array_equal(out[1], _dequant64(wq, s, b, 64, 4)[49].astype(np.float32))


def test_mamba_scan_and_conv_match_loops():
    L, C, NS = 6, 4, 16
    x, dtr, z = (R.round_to(rng.standard_normal((L, C)).astype(np.float32), "float16") for _ in range(3))
    Bm, Cm = (R.round_to(rng.standard_normal((L, NS)).astype(np.float32), "float16") for _ in range(2))
    A = -np.tile(np.arange(1, NS + 1, dtype=np.float32), (C, 1))
    Dv = np.ones(C, np.float32)
    y = R.mamba_scan(x, dtr, None, A, Bm, Cm, Dv, z)
    h = np.zeros((C, NS))
    for t in range(L):
        dt = np.log1p(np.exp(dtr[t].astype(np.float64)))
        h = np.exp(dt[:, None] * A) * h + (dt[:, None] * Bm[t][None, :]) * x[t][:, None]
        yt = (h * Cm[t][None, :]).sum(1) + Dv * x[t]
        ref = yt * z[t] / (1 + np.exp(-z[t].astype(np.float64)))
        assert np.abs(y[t] - ref).max() <= 2e-3 * max(1.0, np.abs(ref).max())
    w = R.round_to(rng.standard_normal((C, 4)).astype(np.float32), "float16")
    yc = R.causal_conv1d(x, w, None, None, silu=False)
    for l in range(L):
        acc = sum(w[:, j] * (x[l - 3 + j] if l - 3 + j >= 0 else 0) for j in range(4))
        assert np.abs(yc[l] - acc).max() <= 2e-3 * max(1.0, np.abs(acc).max())


# ------------------------------------------- second oracle path: the MLX-derived header arithmetic
def test_oracle_dequant_equals_mlx_deq8_bit_for_bit():
    """The oracle's dequantisation (round(round(s*q)+b) in bf16) against the
    reference-held mlx_deq8 arithmetic (oracle/mlx_header_ref.py)."""
    from oracle import mlx_header_ref as H
    r = np.random.default_rng(41)
    wq, s, b = R.quantize_affine(r.standard_normal((96, 1024)).astype(np.float32) * 0.02, 64, 4, "bfloat16")
    got = R.dequantize(wq, s, b, 64, 4, "bfloat16")
    want = H.deq8(wq, s, b, 64)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


QMV_HEADER_CASES = [(1, 256, 2560), (2, 128, 4096), (1, 64, 9728)]


@pytest.mark.parametrize("M,N,K", QMV_HEADER_CASES)
def test_oracle_qmv_against_mlx_qdot16(M, N, K):
    """The oracle's qmv (factored form, fp32 sums in its own order) against the
    qmv_qdot16 arithmetic. With the quad sums of x in fp32 the two are the
    same factored form: within one bf16 ulp plus 2^-9 of the row scale. With
    MLX's bf16 quad sums the outputs also differ by that rounding noise:
    within 6 standard deviations of it (quad_sum_sigma) on top."""
    from oracle import mlx_header_ref as H
    r = np.random.default_rng(K + N)
    x = R.round_to(r.standard_normal((M, K)).astype(np.float32), "bfloat16")
    wq, s, b = R.quantize_affine(r.standard_normal((N, K)).astype(np.float32) * 0.02, 64, 4, "bfloat16")
    got = R.qmv(x, wq, s, b, 64, 4, "bfloat16")
    same_form = H.qmv_qdot16(x, wq, s, b, 64, bf16_quad_sums=False)
    tol = 2 ** -7 * np.abs(same_form) + 2 ** -9 * np.abs(same_form).max()
    assert (np.abs(got - same_form) <= tol).all(), np.abs(got - same_form).max()
    mlx = H.qmv_qdot16(x, wq, s, b, 64)
    tol = 2 ** -7 * np.abs(mlx) + 2 ** -9 * np.abs(mlx).max() + 6 * H.quad_sum_sigma(x, b, 64)
    assert (np.abs(got - mlx) <= tol).all(), np.abs(got - mlx).max()
