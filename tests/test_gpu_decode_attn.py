"""Fused decode attention (mt_qk_norm_rope_sdpa_decode): the caches it writes
are bit-identical to mt_qk_norm_rope_cache's, and its output matches the
two-launch path (mt_qk_norm_rope_cache -> mt_sdpa) and the oracle's
composition of the same two regions within the SDPA tolerance (the keys are
split across warps, so the softmax sums run in another order)."""
import math

import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

pytestmark = pytest.mark.gpu

EPS, THETA = 1e-6, 1e6


def t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype).cuda()


def n(x):
    return x.float().cpu().numpy()


def close(got, ref, *, ulps, abs_frac):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    tol = ulps * 2 ** -7 * np.abs(ref) + abs_frac * max(np.abs(ref).max(), 1e-30)
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {np.abs(got - ref).max():.4g}"


CASES = [
    # T, Hq, Hkv, offset, cache rows, dtype
    (1, 32, 8, 128, 160, "bfloat16"),  # Qwen3-4B decode after a 128-token prefill
    (2, 16, 4, 77, 96, "bfloat16"),
    (4, 8, 2, 0, 8, "bfloat16"),  # decode into an empty cache
    (1, 32, 8, 2047, 2048, "bfloat16"),  # long context: 64 key blocks over 8 warps
    (3, 4, 4, 300, 320, "bfloat16"),  # one query head per kv head
    (1, 8, 2, 50, 64, "float16"),
]


@pytest.mark.parametrize("T,Hq,Hkv,offset,cap,dtype", CASES)
def test_decode_attention(cuda, oracle, T, Hq, Hkv, offset, cap, dtype):
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    D = 128
    r = np.random.default_rng(T * 1000 + offset)
    rd = lambda *s: oracle.round_to(r.standard_normal(s).astype(np.float32), dtype)
    q, k, v = rd(T, Hq * D), rd(T, Hkv * D), rd(T, Hkv * D)
    qw = oracle.round_to(1.0 + 0.2 * r.standard_normal(D).astype(np.float32), dtype)
    kw = oracle.round_to(1.0 + 0.2 * r.standard_normal(D).astype(np.float32), dtype)
    kc0, vc0 = rd(Hkv, cap, D), rd(Hkv, cap, D)
    scale = 1.0 / math.sqrt(D)

    kc1, vc1 = t(kc0, tdt), t(vc0, tdt)
    o1 = lib.qk_norm_rope_sdpa_decode(t(q, tdt), t(k, tdt), t(v, tdt), t(qw, tdt), t(kw, tdt), EPS, kc1, vc1,
                                      n_heads=Hq, n_kv_heads=Hkv, offset=offset, rope_base=THETA, scale=scale)
    kc2, vc2 = t(kc0, tdt), t(vc0, tdt)
    qh = torch.empty(Hq, T, D, dtype=tdt, device="cuda")
    lib.qk_norm_rope_cache(t(q, tdt), t(k, tdt), t(v, tdt), t(qw, tdt), t(kw, tdt), EPS, qh, kc2, vc2,
                           n_heads=Hq, n_kv_heads=Hkv, offset=offset, rope_base=THETA)
    L = offset + T
    o2 = lib.sdpa(qh[None], kc2[None, :, :L], vc2[None, :, :L], scale=scale, causal=True, q_offset=offset,
                  out_layout="blhd").reshape(T, Hq * D)
    torch.cuda.synchronize()
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    close(n(o1), n(o2), ulps=2, abs_frac=2 ** -8)

    kc3, vc3 = kc0.copy(), vc0.copy()
    qo, kc3, vc3 = oracle.qk_norm_rope_cache(q, k, v, qw, kw, EPS, kc3, vc3, Hq, Hkv, offset, THETA, dtype)
    ref = oracle.sdpa(qo[None], kc3[None, :, :L], vc3[None, :, :L], scale, True, offset, dtype)
    ref = ref[0].transpose(1, 0, 2).reshape(T, Hq * D)
    close(n(o1), ref, ulps=2 if dtype == "bfloat16" else 8, abs_frac=2 ** -8)


def test_decode_attention_refuses_prefill_rows(cuda):
    """More than 16 query rows per kv head is the prefill path's: reported, nothing written."""
    T, Hq, Hkv, D = 5, 32, 8, 128
    q = torch.zeros(T, Hq * D, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(T, Hkv * D, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    kc = torch.full((Hkv, 16, D), 3.0, dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    with pytest.raises(lib.MTError, match="at most 4 tokens"):
        lib.qk_norm_rope_sdpa_decode(q, k, k, w, w, EPS, kc, vc, n_heads=Hq, n_kv_heads=Hkv, offset=0,
                                     rope_base=THETA, scale=0.1)
    assert bool((kc == 3.0).all()) and bool((vc == 3.0).all())
