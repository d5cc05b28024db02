"""Parity of every libmt kernel with the CPU oracle on seeded inputs.

Tolerances (stated per test): integer/byte/index work and fixed-order
arithmetic are compared bit for bit; reordered fp32 sums rounded to bf16 are
allowed one bf16 ulp of the reference (2^-7 relative) plus an absolute term
of 2^-9 * max|ref| that covers summation-order differences on outputs near
zero."""
import math

import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

pytestmark = pytest.mark.gpu

rng = np.random.default_rng(1234)
BF = torch.bfloat16


def t(a, dtype=BF):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype).cuda()


def n(x: torch.Tensor) -> np.ndarray:
    return x.float().cpu().numpy()


def close_bf16(got, ref, *, ulps=1, abs_frac=2 ** -9):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    tol = ulps * 2 ** -7 * np.abs(ref) + abs_frac * max(np.abs(ref).max(), 1e-30)
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {np.abs(got - ref).max():.4g}"


def quantized(oracle, N, K, group=64, bits=4, dtype="bfloat16", seed=0):
    r = np.random.default_rng(seed)
    wq, s, b = oracle.quantize_affine(r.standard_normal((N, K)).astype(np.float32) * 0.02, group, bits, dtype)
    tdt = BF if dtype == "bfloat16" else torch.float16
    return (wq, s, b), (torch.from_numpy(wq.view(np.int32)).cuda(), t(s, tdt), t(b, tdt))


# --------------------------------------------------------------- quantized matmul
QMM_CASES = [
    # M, N, K, group, bits, dtype
    (1, 512, 512, 64, 4, "bfloat16"),
    (3, 300, 1024, 64, 4, "bfloat16"),
    (8, 256, 2560, 64, 4, "bfloat16"),
    (1, 256, 512, 64, 8, "bfloat16"),
    (1, 256, 512, 32, 4, "float16"),
    (16, 256, 512, 64, 4, "bfloat16"),
    (127, 384, 2560, 64, 4, "bfloat16"),
    (128, 1024, 2560, 64, 4, "bfloat16"),
    (200, 256, 1024, 128, 4, "bfloat16"),
    (130, 200, 576, 64, 4, "bfloat16"),
    (64, 256, 1024, 64, 8, "bfloat16"),
    (96, 256, 1024, 64, 4, "float16"),
    (512, 256, 512, 64, 4, "bfloat16"),
    # decode shapes of Qwen3-4B (streamed qmv): down, o_proj, a wide projection, 2 rows of x
    (1, 2560, 9728, 64, 4, "bfloat16"),
    (1, 2560, 4096, 64, 4, "bfloat16"),
    (1, 20000, 2560, 64, 4, "bfloat16"),
    (1, 151936, 2560, 64, 4, "bfloat16"),  # lm_head rows: scales streamed with the weight stages
    (2, 1536, 2560, 64, 4, "float16"),
]


@pytest.mark.parametrize("M,N,K,group,bits,dtype", QMM_CASES)
def test_quantized_matmul(cuda, oracle, M, N, K, group, bits, dtype):
    tdt = BF if dtype == "bfloat16" else torch.float16
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), dtype)
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, N, K, group, bits, dtype)
    y = lib.quantized_matmul(t(x, tdt), wq_t, s_t, b_t, group_size=group, bits=bits)
    torch.cuda.synchronize()
    ref = oracle.quantized_matmul(x, wq, s, b, group, bits, dtype)
    close_bf16(n(y), ref, ulps=1 if dtype == "bfloat16" else 8)


@pytest.mark.parametrize("M", [1, 128])
def test_quantized_matmul_residual_and_norm(cuda, oracle, M):
    N, K = 256, 1024
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    r = oracle.round_to(rng.standard_normal((M, N)).astype(np.float32), "bfloat16")
    w = oracle.round_to(rng.standard_normal(N).astype(np.float32), "bfloat16")
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, N, K)
    y = lib.quantized_matmul(t(x), wq_t, s_t, b_t, residual=t(r))
    ref = oracle.add(oracle.quantized_matmul(x, wq, s, b), r)
    close_bf16(n(y), ref, ulps=2)
    h, yn = lib.quantized_matmul_residual_rms_norm(t(x), wq_t, s_t, b_t, t(r), t(w), 1e-6)
    close_bf16(n(h), ref, ulps=2)
    close_bf16(n(yn), oracle.rms_norm(n(h), w, 1e-6), ulps=1)


@pytest.mark.parametrize("M", [1, 5, 128, 160])
def test_quantized_matmul_swiglu(cuda, oracle, M):
    N, K = 384, 1024
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    (wg, sg, bg), gt = quantized(oracle, N, K, seed=1)
    (wu, su, bu), ut = quantized(oracle, N, K, seed=2)
    y = lib.quantized_matmul_swiglu(t(x), *gt, *ut)
    g = oracle.quantized_matmul(x, wg, sg, bg)
    u = oracle.quantized_matmul(x, wu, su, bu)
    close_bf16(n(y), oracle.swiglu(g, u), ulps=3, abs_frac=2 ** -8)


@pytest.mark.parametrize("M", [1, 128])
def test_quantized_matmul_multi(cuda, oracle, M):
    K = 1024
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    sets = [quantized(oracle, Nn, K, seed=10 + i) for i, Nn in enumerate((512, 128, 200))]
    ys = lib.quantized_matmul_multi(t(x), [g for _, g in sets])
    for (wq, s, b), _ in sets:
        pass
    for ((wq, s, b), _), y in zip(sets, ys):
        close_bf16(n(y), oracle.quantized_matmul(x, wq, s, b), ulps=1)


def test_split_k_is_deterministic(cuda, oracle):
    """Split-K partials are summed in split order: three runs are bitwise equal."""
    M, N, K = 128, 512, 4096
    x = t(oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16"))
    _, (wq_t, s_t, b_t) = quantized(oracle, N, K)
    outs = [lib.quantized_matmul(x, wq_t, s_t, b_t) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))


def test_qmm_device_status_clean(cuda):
    assert lib.device_status(clear=True) == 0


# --------------------------------------------------------------- norms / rope
@pytest.mark.parametrize("rows,dim", [(1, 2560), (128, 2560), (7, 100), (3, 4096)])
def test_rms_norm(cuda, oracle, rows, dim):
    x = oracle.round_to(rng.standard_normal((rows, dim)).astype(np.float32), "bfloat16")
    w = oracle.round_to(rng.standard_normal(dim).astype(np.float32), "bfloat16")
    y = lib.rms_norm(t(x), t(w), 1e-6)
    close_bf16(n(y), oracle.rms_norm(x, w, 1e-6), ulps=1, abs_frac=0)
    r = oracle.round_to(rng.standard_normal((rows, dim)).astype(np.float32), "bfloat16")
    h, yy = lib.add_rms_norm(t(x), t(r), t(w), 1e-6)
    hr, yr = oracle.add_rms_norm(x, r, w, 1e-6)
    assert np.array_equal(n(h), hr)  # the add is exact elementwise work
    close_bf16(n(yy), yr, ulps=1, abs_frac=0)


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_layer_norm(cuda, oracle, dtype):
    tdt = torch.float16 if dtype == "float16" else torch.float32
    x = oracle.round_to(rng.standard_normal((33, 1280)).astype(np.float32), dtype)
    w = oracle.round_to(rng.standard_normal(1280).astype(np.float32), dtype)
    b = oracle.round_to(rng.standard_normal(1280).astype(np.float32), dtype)
    y = lib.layer_norm(t(x, tdt), t(w, tdt), t(b, tdt), 1e-5)
    ref = oracle.layer_norm(x, w, b, 1e-5, dtype)
    tol = (2 ** -10 if dtype == "float16" else 1e-5)
    assert np.abs(n(y) - ref).max() <= tol * np.abs(ref).max() + 1e-4


@pytest.mark.parametrize("dims,traditional,offset", [(128, False, 0), (128, False, 128), (64, True, 5),
                                                     (96, False, 2047)])
def test_rope(cuda, oracle, dims, traditional, offset):
    x = oracle.round_to(rng.standard_normal((4, 9, 128)).astype(np.float32), "bfloat16")
    y = lib.rope(t(x), dims, traditional=traditional, base=1e6, offset=offset)
    ref = oracle.rope(x, dims, traditional, 1e6, 1.0, offset)
    close_bf16(n(y), ref, ulps=1, abs_frac=2 ** -10)
    assert np.array_equal(n(y)[..., dims:], x[..., dims:])


@pytest.mark.parametrize("T,offset", [(128, 0), (1, 128), (5, 17)])
def test_qk_norm_rope_cache(cuda, oracle, T, offset):
    Hq, Hkv, D, cap = 8, 2, 128, 160
    q = oracle.round_to(rng.standard_normal((T, Hq * D)).astype(np.float32), "bfloat16")
    k = oracle.round_to(rng.standard_normal((T, Hkv * D)).astype(np.float32), "bfloat16")
    v = oracle.round_to(rng.standard_normal((T, Hkv * D)).astype(np.float32), "bfloat16")
    qw = oracle.round_to(rng.standard_normal(D).astype(np.float32), "bfloat16")
    kw = oracle.round_to(rng.standard_normal(D).astype(np.float32), "bfloat16")
    kc = torch.zeros(Hkv, cap, D, dtype=BF, device="cuda")
    vc = torch.zeros_like(kc)
    qo = torch.empty(Hq, T, D, dtype=BF, device="cuda")
    lib.qk_norm_rope_cache(t(q), t(k), t(v), t(qw), t(kw), 1e-6, qo, kc, vc, n_heads=Hq, n_kv_heads=Hkv,
                           offset=offset, rope_base=1e6)
    kcr = np.zeros((Hkv, cap, D), np.float32)
    vcr = np.zeros((Hkv, cap, D), np.float32)
    qr, kcr, vcr = oracle.qk_norm_rope_cache(q, k, v, qw, kw, 1e-6, kcr, vcr, Hq, Hkv, offset, 1e6)
    close_bf16(n(qo), qr, ulps=1, abs_frac=2 ** -10)
    close_bf16(n(kc), kcr, ulps=1, abs_frac=2 ** -10)
    assert np.array_equal(n(vc), vcr)


# --------------------------------------------------------------- attention
@pytest.mark.parametrize("B,Hq,Hkv,Lq,Lk,D,causal", [
    (1, 32, 8, 128, 128, 128, True),
    (1, 32, 8, 1, 129, 128, True),
    (2, 4, 4, 70, 70, 64, False),
    (1, 8, 2, 33, 100, 128, True),
    (1, 4, 1, 200, 200, 128, True),
    # decode shapes (a kv head's query rows in one CTA): two tokens, four tokens, long keys, head_dim 64
    (1, 8, 2, 2, 300, 64, True),
    (2, 16, 4, 4, 77, 128, False),
    (1, 4, 4, 3, 1000, 128, True),
    (1, 32, 8, 1, 2048, 128, True),
    # mlx-whisper encoder self-attention for one clip (non-causal MHA, head_dim 64)
    (1, 20, 20, 1500, 1500, 64, False),
    # Llama-3-8B prefill heads over 1024 of its 2048 positions (GQA 32/8)
    (1, 32, 8, 1024, 1024, 128, True),
    # tcgen05 path (from 64 queries and 384 keys): ragged query and key blocks, a chunk of
    # queries after a cached prefix (q_offset = Lk - Lq > 0, the diagonal inside a key block),
    # two clips
    (1, 8, 2, 300, 700, 128, True),
    (2, 4, 4, 129, 513, 64, True),
    (2, 6, 3, 400, 400, 128, False),
])
def test_sdpa(cuda, oracle, B, Hq, Hkv, Lq, Lk, D, causal):
    q = oracle.round_to(rng.standard_normal((B, Hq, Lq, D)).astype(np.float32), "bfloat16")
    k = oracle.round_to(rng.standard_normal((B, Hkv, Lk, D)).astype(np.float32), "bfloat16")
    v = oracle.round_to(rng.standard_normal((B, Hkv, Lk, D)).astype(np.float32), "bfloat16")
    scale = 1 / math.sqrt(D)
    off = Lk - Lq
    o = lib.sdpa(t(q), t(k), t(v), scale=scale, causal=causal, q_offset=off)
    ref = oracle.sdpa(q, k, v, scale, causal, off)
    # P is rounded to bf16 before P.V: 2^-8 relative per term, plus the output rounding
    assert np.abs(n(o) - ref).max() <= 2 ** -7 * np.abs(ref).max() + 4e-3 * np.abs(v).max()
    # heads-concatenated output layout ([B, Lq, Hq, D]) is the same values
    o2 = lib.sdpa(t(q), t(k), t(v), scale=scale, causal=causal, q_offset=off, out_layout="blhd")
    assert torch.equal(o2.transpose(1, 2), o)


def test_sdpa_rows_before_every_key(cuda, oracle):
    """q_offset < 0 on the tcgen05 path: the first query blocks see no key at
    all (zeros, as the oracle writes) and sit in the persistent grid's walk
    between blocks that do."""
    B, Hq, Hkv, Lq, Lk, D, off = 1, 4, 2, 400, 384, 128, -200
    q = oracle.round_to(rng.standard_normal((B, Hq, Lq, D)).astype(np.float32), "bfloat16")
    k = oracle.round_to(rng.standard_normal((B, Hkv, Lk, D)).astype(np.float32), "bfloat16")
    v = oracle.round_to(rng.standard_normal((B, Hkv, Lk, D)).astype(np.float32), "bfloat16")
    o = lib.sdpa(t(q), t(k), t(v), scale=1 / math.sqrt(D), causal=True, q_offset=off)
    ref = oracle.sdpa(q, k, v, 1 / math.sqrt(D), True, off)
    assert not np.any(n(o)[:, :, :-off])  # rows 0..199 see no key
    assert np.abs(n(o) - ref).max() <= 2 ** -7 * np.abs(ref).max() + 4e-3 * np.abs(v).max()


# --------------------------------------------------------------- elementwise / gather
def test_swiglu(cuda, oracle):
    g = oracle.round_to(rng.standard_normal(10001).astype(np.float32) * 4, "bfloat16")
    u = oracle.round_to(rng.standard_normal(10001).astype(np.float32), "bfloat16")
    y = lib.swiglu(t(g), t(u))
    close_bf16(n(y), oracle.swiglu(g, u), ulps=1, abs_frac=0)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_embedding_bit_exact(cuda, oracle, bits, dtype):
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, 1000, 256, 64, bits, dtype)
    tok = np.array([0, 999, 17, 17, 500], np.int32)
    out = lib.quantized_embedding(torch.from_numpy(tok).cuda(), wq_t, s_t, b_t, bits=bits)
    assert np.array_equal(n(out), oracle.quantized_embedding(tok, wq, s, b, 64, bits, dtype))


def test_quantized_embedding_bad_id_reports(cuda, oracle):
    _, (wq_t, s_t, b_t) = quantized(oracle, 10, 128)
    out = lib.quantized_embedding(torch.tensor([3, 12], dtype=torch.int32, device="cuda"), wq_t, s_t, b_t)
    assert lib.device_status(clear=True) != 0
    assert torch.all(out[1] == 0)


def test_logits_pick(cuda, oracle):
    logits = oracle.round_to(rng.standard_normal(151936).astype(np.float32) * 3, "bfloat16")
    tok, lp, lse = lib.logits_pick(t(logits).view(1, -1))
    rt, rlp, rlse = oracle.logits_pick(logits)
    assert int(tok.item()) == rt
    assert abs(float(lse.item()) - rlse) <= 1e-5 * abs(rlse)
    assert abs(float(lp.item()) - rlp) <= 2 * 2 ** -7 * abs(rlp) + 1e-6


def test_linear_tiny_mlp_bit_exact_without_gelu(cuda, oracle):
    """Tiny-MLP shapes: both fp32 linears accumulate k in order with one fused
    multiply-add per term, so the GPU equals the oracle bit for bit."""
    x = rng.standard_normal((32, 256)).astype(np.float32)
    w1 = rng.uniform(-1, 1, (1024, 256)).astype(np.float32) * math.sqrt(6 / 256)
    w2 = rng.uniform(-1, 1, (256, 1024)).astype(np.float32) * math.sqrt(6 / 1024)
    b1 = rng.standard_normal(1024).astype(np.float32) * 0.1
    h = lib.linear(t(x, torch.float32), t(w1, torch.float32), t(b1, torch.float32), act=0)
    assert np.array_equal(n(h), oracle.linear(x, w1, b1, act=0))
    y = lib.linear(h, t(w2, torch.float32), None, act=0)
    assert np.array_equal(n(y), oracle.linear(oracle.linear(x, w1, b1, act=0), w2, None, act=0))


def test_tiny_mlp_with_gelu_within_erf_bounds(cuda, oracle):
    """With GELU the two sides use different erf implementations (CUDA's erff
    on the GPU, <= 2 ulp; glibc's in the oracle, <= 1 ulp). erf's values lie
    in (-1, 1), so each is within 2 * 2^-24 and 2^-24 of the true erf; the
    rounding of x / sqrt(2) moves erf by under 2^-24, and the rounding of
    1 + erf (a value in [0, 2)) by up to 2^-24 on each side. x * (1 + erf) / 2
    then differs by at most |x| * 8 * 2^-25 = |x| * 2^-22 from one side to
    the other, plus the roundings of the final multiply and halving (2 ulp of
    the result each). The output layer then differs by at most sum|w2| times
    the largest hidden difference, plus its own rounding."""
    x = rng.standard_normal((32, 256)).astype(np.float32)
    w1 = rng.uniform(-1, 1, (1024, 256)).astype(np.float32) * math.sqrt(6 / 256)
    w2 = rng.uniform(-1, 1, (256, 1024)).astype(np.float32) * math.sqrt(6 / 1024)
    b1 = np.zeros(1024, np.float32)
    h = lib.linear(t(x, torch.float32), t(w1, torch.float32), t(b1, torch.float32), act=1)
    pre = oracle.linear(x, w1, b1, act=0).astype(np.float64)   # bit-equal on both sides
    h_ref = oracle.linear(x, w1, b1, act=1)
    ulp = np.spacing(np.abs(h_ref).astype(np.float32)).astype(np.float64)
    bound = np.abs(pre) * 2.0 ** -22 + 4 * ulp + 1e-45
    diff = np.abs(n(h).astype(np.float64) - h_ref)
    assert (diff <= bound).all(), (diff - bound).max()
    y = lib.linear(h, t(w2, torch.float32), None, act=0)
    ref = oracle.gelu_mlp(x, w1, b1, w2, None)
    prop = np.abs(w2).sum(axis=1).max() * bound.max()
    assert np.abs(n(y).astype(np.float64) - ref).max() <= 4 * np.spacing(np.float32(np.abs(ref).max())) + prop


def test_gelu_erf_against_double_erf(cuda, oracle):
    """GELU on the GPU (device erff) against a double-precision GELU: within
    CUDA erff's 2-ulp bound plus the rounding of the surrounding fp32 ops."""
    xs = torch.linspace(-6, 6, 100001, device="cuda")
    eye = torch.eye(1, device="cuda")
    g = lib.linear(xs.view(-1, 1).contiguous(), eye, None, act=1).view(-1)
    ref = 0.5 * xs.double() * (1 + torch.erf(xs.double() / math.sqrt(2)))
    bound = 4 * 2 ** -23 * xs.double().abs().clamp(min=1.0)
    assert ((g.double() - ref).abs() <= bound).all()


@pytest.mark.parametrize("dtype,L,NS,decay", [("float16", 64, 16, 1.0), ("bfloat16", 64, 16, 1.0),
                                              ("float16", 512, 16, 1.0), ("float16", 512, 16, 0.002),
                                              ("bfloat16", 300, 16, 0.002), ("float16", 128, 8, 0.002),
                                              ("float16", 257, 32, 0.002)])
def test_mamba_scan(cuda, oracle, dtype, L, NS, decay):
    """Sequential kernel below 128 steps, chunked in time from 128 up (ragged
    chunk ends, an empty last chunk at L=300, the carried-in state). With
    decay 0.002 (A = -0.002 * (1..NS)) a chunk's carry-in still weighs in
    hundreds of steps later, so a wrong carry between chunks shows."""
    tdt = torch.float16 if dtype == "float16" else BF
    C = 96
    x, dtr, z = (oracle.round_to(rng.standard_normal((L, C)).astype(np.float32), dtype) for _ in range(3))
    Bm, Cm = (oracle.round_to(rng.standard_normal((L, NS)).astype(np.float32), dtype) for _ in range(2))
    A = -np.tile(np.arange(1, NS + 1, dtype=np.float32), (C, 1)) * np.float32(decay)
    dtb = (rng.standard_normal(C) * 0.1).astype(np.float32)
    Dv = np.ones(C, np.float32)
    h0 = (rng.standard_normal((C, NS)) * 0.1).astype(np.float32)
    h_gpu = torch.from_numpy(h0.copy()).cuda()
    y = lib.mamba_scan(t(x, tdt), t(dtr, tdt), t(dtb, torch.float32), t(A, torch.float32), t(Bm, tdt), t(Cm, tdt),
                       t(Dv, torch.float32), t(z, tdt), h_state=h_gpu)
    h_ref = h0.copy()
    ref = oracle.mamba_scan(x, dtr, dtb, A, Bm, Cm, Dv, z, h_state=h_ref, dtype=dtype)
    ulp = 2 ** -10 if dtype == "float16" else 2 ** -7
    assert np.abs(n(y) - ref).max() <= 2 * ulp * np.abs(ref).max()
    assert np.abs(h_gpu.cpu().numpy() - h_ref).max() <= 1e-4 * max(1.0, np.abs(h_ref).max())


def test_causal_conv1d_with_state(cuda, oracle):
    L, C, W = 12, 64, 4
    x = oracle.round_to(rng.standard_normal((L, C)).astype(np.float32), "float16")
    w = oracle.round_to(rng.standard_normal((C, W)).astype(np.float32), "float16")
    bias = oracle.round_to(rng.standard_normal(C).astype(np.float32), "float16")
    st = oracle.round_to(rng.standard_normal((C, W - 1)).astype(np.float32), "float16")
    st_gpu = t(st, torch.float16)
    y = lib.causal_conv1d(t(x, torch.float16), t(w, torch.float16), t(bias, torch.float16), conv_state=st_gpu)
    ref = oracle.causal_conv1d(x, w, bias, st, silu=True, dtype="float16")
    assert np.abs(n(y) - ref).max() <= 2 ** -10 * np.abs(ref).max() * 2
    assert np.array_equal(n(st_gpu), x[L - (W - 1):].T)


# --------------------------------------------------------------- output-diff reduction
def _stats(a, b, **kw):
    return lib.read_diff_stats(lib.diff_reduce(a, b, **kw))


@pytest.mark.parametrize("size", [1, 1000, 1 << 20, (1 << 22) + 3])
def test_diff_reduce_matches_contract(cuda, size):
    from oracle import numeric_ref as NR
    ref = rng.standard_normal(size).astype(np.float32)
    cand = ref + rng.standard_normal(size).astype(np.float32) * 1e-3
    if size > 10:
        cand[size // 3] += 0.5
        ref[7] = np.nan
        cand[7] = np.nan
    s = _stats(t(cand, torch.float32), t(ref, torch.float32), rtol=1e-3, atol=1e-3)
    r = NR.compare(cand, ref, 1e-3, 1e-3)
    assert s.nonfinite_violations == 0 and s.nan_excess == 0
    assert (s.max_excess <= 0) == r["passed"]
    assert np.float32(s.max_excess) == np.float32(r["max_excess"])
    assert s.excess_index == int(np.ravel_multi_index(r["index"], cand.shape))
    assert s.over_count == r.get("over", 0)
    assert s.max_abs == pytest.approx(NR.max_abs_diff(cand, ref), rel=0, abs=0)


@pytest.mark.parametrize("dtype", [BF, torch.float16])
@pytest.mark.parametrize("rtol", [1e-2, 2.0])
def test_diff_reduce_16bit_equals_its_fp32_upcast(cuda, dtype, rtol):
    """A 16-bit pair is visited 8 elements at a time (packed checks, the
    finite branch of the policy); its fp32 upcast takes the element-by-
    element policy. Every statistic but the cosine sums must be identical:
    Inf / NaN spread over some vectors, +0 vs -0, equal and unequal vectors,
    the largest finite magnitudes (with rtol 2 their allowed error and
    |a - b| both overflow: the scaled form) and a ragged tail."""
    n = 8 * 4099 + 5
    g = torch.Generator(device="cuda").manual_seed(11)
    b = torch.randn(n, generator=g, device="cuda")
    a = b + torch.randn(n, generator=g, device="cuda") * 0.05
    a[:64] = b[:64]                                       # whole equal vectors
    big = torch.finfo(dtype).max
    a[100], b[100] = 0.0, -0.0                             # bits differ, values equal
    a[205], b[205] = float("inf"), float("inf")
    a[317], b[317] = float("nan"), 1.0                     # a non-finite where b is finite
    a[333], b[333] = 2.0, float("-inf")
    a[900], b[900] = big, -big                             # |a - b| overflows fp32 for bf16
    a[901], b[901] = -big, big
    a[n - 2] = float("nan")                                # in the tail
    a16, b16 = a.to(dtype), b.to(dtype)
    s16 = _stats(a16, b16, rtol=rtol, atol=1e-3)
    s32 = _stats(a16.float(), b16.float(), rtol=rtol, atol=1e-3)
    for f in ("max_excess", "excess_index", "over_count", "nonfinite_violations", "first_violation",
              "nan_excess", "max_abs", "amax_a", "amax_b"):
        assert getattr(s16, f) == getattr(s32, f), f
    # bit mismatches of the 16-bit values (the fp32 upcast keeps them one for one)
    diff = (a16.view(torch.int16) != b16.view(torch.int16)).cpu().numpy()
    assert s16.bit_mismatches == s32.bit_mismatches == int(diff.sum())
    assert s16.first_mismatch == s32.first_mismatch == int(np.argmax(diff))
    for f in ("dot_ab", "dot_aa", "dot_bb"):
        assert getattr(s16, f) == pytest.approx(getattr(s32, f), rel=1e-6), f


def test_numeric_compare_on_golden_cases(cuda):
    from metal_autotune_b200.autotuner_runtime import numeric
    from tests.conftest import fval, golden
    G = golden("numeric_contract.json")
    for name in ("within_tolerance", "worst_offender", "wobble_rescues", "candidate_nonfinite",
                 "reference_nonfinite_same", "reference_nonfinite_wrong_sign", "reference_nonfinite_finite_for_nan"):
        c = G["ladder"][name]
        r = numeric.compare(torch.tensor(fval(c["candidate"])).cuda(), torch.tensor(fval(c["reference"])).cuda(),
                            c.get("rtol", 0.0), c.get("atol", 0.0), c.get("wobble", 0.0))
        assert r.passed is c["passed"], name
        if "reason" in c:
            assert r.reason == c["reason"]
        if "index" in c:
            assert r.index == tuple(c["index"])
    for ref, cand, exact, passed in G["cases"]["test_shared_policy_exact_and_tolerance"]["rows"]:
        r = numeric.check(torch.tensor(fval(cand)).cuda(), torch.tensor(fval(ref)).cuda(), exact=exact,
                          rtol=0.01, atol=0.001)
        assert r.passed is passed
    ov = G["cases"]["test_tolerance_cannot_hide_extreme_subtraction_overflow"]
    for e in ov["expect"]:
        r = numeric.check(torch.tensor(ov["candidate"]).cuda(), torch.tensor(ov["reference"]).cuda(), exact=False,
                          rtol=e["rtol"], atol=e["atol"])
        assert r.passed is e["passed"]
    bad = torch.tensor([2 ** 24 + 1], dtype=torch.int32).cuda()
    assert not numeric.compare(bad, torch.tensor([2 ** 24], dtype=torch.int32).cuda(), 1.0, 100.0).passed


def test_bitwise_and_cosine(cuda):
    from metal_autotune_b200.autotuner_runtime import exact, numeric
    from oracle import numeric_ref as NR
    a = torch.randn(5000, device="cuda").to(BF)
    assert exact.bitwise_equal(a, a.clone())
    b = a.clone()
    b[123] = -b[123] if b[123] != 0 else 1
    assert not exact.bitwise_equal(a, b)
    z = torch.zeros(4, device="cuda")
    assert not exact.bitwise_equal(z, -z)
    c = numeric.cosine(a, b)
    assert c == pytest.approx(NR.cosine(n(a), n(b)), abs=1e-6)


# --------------------------------------------------------------- conv1d (Whisper conv stem)
CONV_CASES = [
    # N, L, Cin, Cout, K, stride, padding, act, bias, dtype
    (1, 40, 32, 64, 3, 1, 1, 0, False, "float16"),
    (2, 301, 128, 256, 3, 1, 1, 1, True, "float16"),       # conv1 form, odd length
    (1, 300, 256, 192, 3, 2, 1, 1, True, "bfloat16"),      # conv2 form, Cout not a multiple of 128
    (1, 50, 64, 129, 3, 1, 1, 0, True, "bfloat16"),        # odd Cout: scalar tail stores
    (1, 3000, 128, 1280, 3, 1, 1, 1, True, "float16"),     # mlx-whisper conv1 at full length
    (1, 600, 1280, 1280, 3, 2, 1, 1, True, "float16"),     # conv2 channels, shortened
    (2, 3000, 1280, 1280, 3, 2, 1, 1, True, "float16"),    # mlx-whisper conv2 at full length, two clips
    (3, 200, 128, 256, 3, 1, 1, 1, True, "bfloat16"),      # several clips, row tiles ending mid-clip
    (1, 301, 128, 128, 3, 2, 1, 1, True, "float16"),       # stride 2 over an odd length (mma.sync path)
    (2, 64, 64, 64, 4, 1, 2, 0, False, "bfloat16"),        # 4 taps, padding 2
]


@pytest.mark.parametrize("N,L,Cin,Cout,K,stride,pad,act,bias,dtype", CONV_CASES)
def test_conv1d(cuda, oracle, N, L, Cin, Cout, K, stride, pad, act, bias, dtype):
    tdt = BF if dtype == "bfloat16" else torch.float16
    r = np.random.default_rng(L + Cout)
    x = oracle.round_to(r.standard_normal((N, L, Cin)).astype(np.float32), dtype)
    w = oracle.round_to(r.standard_normal((Cout, K, Cin)).astype(np.float32) / np.sqrt(K * Cin), dtype)
    b = oracle.round_to(r.standard_normal(Cout).astype(np.float32) * 0.1, dtype) if bias else None
    y = lib.conv1d(t(x, tdt), t(w, tdt), t(b, tdt) if bias else None, stride=stride, padding=pad, act=act)
    torch.cuda.synchronize()
    ref = oracle.conv1d(x, w, b, stride, pad, act, dtype)
    assert tuple(y.shape) == ref.shape
    # fp32 sums in another order than the oracle's sequential one: a rounding
    # step of the element type at most, after each of conv / bias / GELU
    ulp = 2.0 ** (-7 if dtype == "bfloat16" else -10)
    got, refd = n(y).astype(np.float64), ref.astype(np.float64)
    tol = 3 * ulp * np.abs(refd) + 2 * ulp * np.abs(refd).max()
    bad = np.abs(got - refd) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {np.abs(got - refd).max():.4g}"


# --------------------------------------------------------------- 16-bit linear (Whisper MLP)
@pytest.mark.parametrize("M,N,K,act,bias,dtype", [
    (100, 320, 256, 1, True, "float16"),
    (37, 130, 64, 0, False, "bfloat16"),
    (1500, 5120, 1280, 1, True, "float16"),   # mlx-whisper fc1 for one 1500-frame clip
    (1500, 1280, 5120, 0, True, "float16"),   # fc2
    (200, 256, 200, 0, True, "bfloat16"),     # K not a multiple of 64: zero-filled tail block
    (512, 96, 2048, 0, False, "float16"),     # Mamba-370m x_proj (N = dt_rank + 2 d_state)
    (512, 4096, 1024, 0, False, "float16"),   # Mamba-370m in_proj
    (512, 2048, 64, 0, True, "float16"),      # Mamba-370m dt_proj
])
def test_linear_16bit(cuda, oracle, M, N, K, act, bias, dtype):
    tdt = BF if dtype == "bfloat16" else torch.float16
    r = np.random.default_rng(M + N + K)
    x = oracle.round_to(r.standard_normal((M, K)).astype(np.float32), dtype)
    w = oracle.round_to(r.standard_normal((N, K)).astype(np.float32) / np.sqrt(K), dtype)
    b = oracle.round_to(r.standard_normal(N).astype(np.float32) * 0.1, dtype) if bias else None
    y = lib.linear(t(x, tdt), t(w, tdt), t(b, tdt) if bias else None, act=act)
    torch.cuda.synchronize()
    ref = oracle.linear_lp(x, w, b, act, dtype)
    ulp = 2.0 ** (-7 if dtype == "bfloat16" else -10)
    got, refd = n(y).astype(np.float64), ref.astype(np.float64)
    tol = 3 * ulp * np.abs(refd) + 2 * ulp * np.abs(refd).max()
    bad = np.abs(got - refd) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {np.abs(got - refd).max():.4g}"


@pytest.mark.parametrize("M,N,K,bias,dtype", [(300, 1280, 1280, True, "float16"), (129, 200, 512, False, "bfloat16"),
                                             (1500, 1280, 5120, True, "float16")])
def test_linear_residual(cuda, oracle, M, N, K, bias, dtype):
    """x + linear(h): round(round(h w^T + b) + x), the residual branch of the
    mlx-whisper blocks, against the oracle's linear then add."""
    tdt = BF if dtype == "bfloat16" else torch.float16
    r = np.random.default_rng(M * 3 + N + K)
    h = oracle.round_to(r.standard_normal((M, K)).astype(np.float32), dtype)
    w = oracle.round_to(r.standard_normal((N, K)).astype(np.float32) / np.sqrt(K), dtype)
    b = oracle.round_to(r.standard_normal(N).astype(np.float32) * 0.1, dtype) if bias else None
    x = oracle.round_to(r.standard_normal((M, N)).astype(np.float32), dtype)
    y = lib.linear_residual(t(h, tdt), t(w, tdt), t(b, tdt) if bias else None, t(x, tdt))
    ref = oracle.add(oracle.linear_lp(h, w, b, 0, dtype), x, dtype)
    ulp = 2.0 ** (-7 if dtype == "bfloat16" else -10)
    got, refd = n(y).astype(np.float64), ref.astype(np.float64)
    tol = 3 * ulp * np.abs(refd) + 2 * ulp * np.abs(refd).max()
    bad = np.abs(got - refd) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {np.abs(got - refd).max():.4g}"
