"""TEST INFRASTRUCTURE — numpy front end of the CPU oracle (liboracle.so).

Arrays are float32 holding values representable in the region's element type
(bf16/fp16 inputs are passed as their exact float32 values); results come
back as float32 arrays of element-type values. Only tests/, smoke() and the
bench's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .build import build_oracle

DT = {"bfloat16": 0, "float16": 1, "float32": 2}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = C.CDLL(str(build_oracle()))
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        I64, I, F = C.c_int64, C.c_int, C.c_float
        sig = {
            "orc_round": (F, [F, I]),
            "orc_qmm_t": (None, [f32p, u32p, f32p, f32p, f32p, I64, I64, I64, I, I, I]),
            "orc_qmv": (None, [f32p, u32p, f32p, f32p, f32p, I64, I64, I64, I, I, I]),
            "orc_rms_norm": (None, [f32p, f32p, F, f32p, I64, I64, I]),
            "orc_layer_norm": (None, [f32p, C.c_void_p, C.c_void_p, F, f32p, I64, I64, I]),
            "orc_rope": (None, [f32p, f32p, I64, I64, I64, I, I, F, F, I64, I]),
            "orc_qk_norm_rope_cache": (None, [f32p, f32p, f32p, f32p, f32p, F, f32p, f32p, f32p, I64, I64, I64,
                                              I64, I64, I64, F, I]),
            "orc_swiglu": (None, [f32p, f32p, f32p, I64, I]),
            "orc_sdpa": (None, [f32p, f32p, f32p, f32p, I64, I64, I64, I64, I64, I64, F, I, I64, I]),
            "orc_quantized_embedding": (None, [i32p, u32p, f32p, f32p, f32p, I64, I64, I64, I, I, I]),
            "orc_logits_pick": (None, [f32p, I64, I, C.POINTER(C.c_int32), C.POINTER(F), C.POINTER(F)]),
            "orc_linear": (None, [f32p, f32p, C.c_void_p, f32p, I64, I64, I64, I]),
            "orc_erf": (F, [F]),
            "orc_gelu": (F, [F]),
            "orc_mamba_scan": (None, [f32p, f32p, C.c_void_p, f32p, f32p, f32p, C.c_void_p, f32p, f32p,
                                      C.c_void_p, I64, I64, I64, I]),
            "orc_causal_conv1d": (None, [f32p, f32p, C.c_void_p, C.c_void_p, f32p, I64, I64, I, I, I]),
            "orc_conv1d": (None, [f32p, f32p, C.c_void_p, f32p, I64, I64, I64, I64, I, I, I, I, I]),
            "orc_linear_lp": (None, [f32p, f32p, C.c_void_p, f32p, I64, I64, I64, I, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _opt(a):
    return None if a is None else _f32(a).ctypes.data_as(C.c_void_p)


# ------------------------------------------------------------- element types
def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even, NaN kept quiet."""
    u = _f32(a).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(a, dtype: str) -> np.ndarray:
    a = _f32(a)
    if dtype == "bfloat16":
        return bf16_value(bf16_bits(a))
    if dtype == "float16":
        return a.astype(np.float16).astype(np.float32)
    return a.copy()


# ------------------------------------------------------------- quantiser
def quantize_affine(w: np.ndarray, group: int = 64, bits: int = 4, dtype: str = "bfloat16"):
    """MLX-style affine quantisation of w [N, K] per group of `group` values
    along K: scale = (max-min)/(2^bits-1), bias = min, q = round((w-bias)/scale)
    clipped to [0, 2^bits-1]; scale and bias rounded to `dtype`; values packed
    little-end-first into uint32 words (value j of a word at bits
    [j*bits, (j+1)*bits), autotuner/scaffold/lower.py:1207-1212).
    Returns (wq uint32 [N, K*bits/32], scales, biases) with scales/biases as
    float32 arrays of `dtype` values."""
    w = _f32(w)
    N, K = w.shape
    G = K // group
    levels = (1 << bits) - 1
    g = w.reshape(N, G, group)
    lo, hi = g.min(axis=2), g.max(axis=2)
    scale = np.maximum((hi - lo) / levels, 1e-8).astype(np.float32)
    scale = round_to(scale, dtype)
    bias = round_to(lo, dtype)
    q = np.clip(np.rint((g - bias[..., None]) / scale[..., None]), 0, levels).astype(np.uint32).reshape(N, K)
    per = 32 // bits
    q = q.reshape(N, K // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    wq = np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)
    return np.ascontiguousarray(wq), scale, bias


def unpack(wq: np.ndarray, bits: int) -> np.ndarray:
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    q = (wq[:, :, None] >> shifts) & ((1 << bits) - 1)
    return q.reshape(wq.shape[0], -1)


# ------------------------------------------------------------- regions
def qmm_t(x, wq, scales, biases, group=64, bits=4, dtype="bfloat16"):
    x = _f32(x)
    K = x.shape[-1]
    M = x.size // K
    N = wq.shape[0]
    y = np.empty((M, N), np.float32)
    lib().orc_qmm_t(x.reshape(M, K), np.ascontiguousarray(wq, np.uint32), _f32(scales), _f32(biases), y, M, N, K,
                    group, bits, DT[dtype])
    return y.reshape(*x.shape[:-1], N)


def qmv(x, wq, scales, biases, group=64, bits=4, dtype="bfloat16"):
    x = _f32(x)
    K = x.shape[-1]
    M = x.size // K
    N = wq.shape[0]
    y = np.empty((M, N), np.float32)
    lib().orc_qmv(x.reshape(M, K), np.ascontiguousarray(wq, np.uint32), _f32(scales), _f32(biases), y, M, N, K,
                  group, bits, DT[dtype])
    return y.reshape(*x.shape[:-1], N)


QMV_MAX_ROWS = 8


def quantized_matmul(x, wq, scales, biases, group=64, bits=4, dtype="bfloat16"):
    """The library's dispatch: qmv below the batch limit, qmm_t above
    (autotuner/scaffold/stitch.py:74-89; this build's limit is 8 rows)."""
    M = np.asarray(x).size // np.asarray(x).shape[-1]
    f = qmv if M <= QMV_MAX_ROWS else qmm_t
    return f(x, wq, scales, biases, group, bits, dtype)


def rms_norm(x, w, eps, dtype="bfloat16"):
    x = _f32(x)
    D = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_rms_norm(x, _f32(w), eps, y, x.size // D, D, DT[dtype])
    return y


def add(x, r, dtype="bfloat16"):
    return round_to(_f32(x) + _f32(r), dtype)


def add_rms_norm(x, r, w, eps, dtype="bfloat16"):
    h = add(x, r, dtype)
    return h, rms_norm(h, w, eps, dtype)


def layer_norm(x, w, b, eps, dtype="float16"):
    x = _f32(x)
    D = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_layer_norm(x, _opt(w), _opt(b), eps, y, x.size // D, D, DT[dtype])
    return y


def rope(x, dims, traditional=False, base=10000.0, scale=1.0, offset=0, dtype="bfloat16"):
    x = _f32(x)
    L, D = x.shape[-2], x.shape[-1]
    R = x.size // (L * D)
    y = np.empty_like(x)
    lib().orc_rope(x, y, R, L, D, dims, int(traditional), base, scale, offset, DT[dtype])
    return y


def qk_norm_rope_cache(q, k, v, qw, kw, eps, k_cache, v_cache, Hq, Hkv, offset, base, dtype="bfloat16"):
    """Returns (q_out [Hq, T, D], k_cache, v_cache) with the caches updated in place."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    T = q.shape[0]
    D = q.shape[1] // Hq
    if offset < 0 or offset + T > k_cache.shape[-2] or v_cache.shape != k_cache.shape:
        raise ValueError(f"cache rows {offset}..{offset + T} outside a cache of {k_cache.shape[-2]}")
    for c in (k_cache, v_cache):
        if c.dtype != np.float32 or not c.flags.c_contiguous:
            raise ValueError("caches must be C-contiguous float32 (updated in place)")
    q_out = np.zeros((Hq, T, D), np.float32)
    lib().orc_qk_norm_rope_cache(q, k, v, _f32(qw), _f32(kw), eps, q_out, k_cache, v_cache, T, Hq, Hkv, D,
                                 k_cache.shape[-2], offset, base, DT[dtype])
    return q_out, k_cache, v_cache


def swiglu(g, u, dtype="bfloat16"):
    g, u = _f32(g), _f32(u)
    y = np.empty_like(g)
    lib().orc_swiglu(g, u, y, g.size, DT[dtype])
    return y


def sdpa(q, k, v, scale, causal, q_offset=0, dtype="bfloat16"):
    """q [B,Hq,Lq,D], k/v [B,Hkv,Lk,D] -> o [B,Hq,Lq,D]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hq, Lq, D = q.shape
    Hkv, Lk = k.shape[1], k.shape[2]
    o = np.empty_like(q)
    lib().orc_sdpa(q, k, v, o, B, Hq, Hkv, Lq, Lk, D, scale, int(causal), q_offset, DT[dtype])
    return o


def quantized_embedding(tokens, wq, scales, biases, group=64, bits=4, dtype="bfloat16"):
    tok = np.ascontiguousarray(tokens, np.int32).reshape(-1)
    D = wq.shape[1] * (32 // bits)
    out = np.empty((tok.size, D), np.float32)
    lib().orc_quantized_embedding(tok, np.ascontiguousarray(wq, np.uint32), _f32(scales), _f32(biases), out,
                                  tok.size, wq.shape[0], D, group, bits, DT[dtype])
    return out.reshape(*np.shape(tokens), D)


def dequantize(wq, scales, biases, group=64, bits=4, dtype="bfloat16"):
    """The dequantised weight matrix [N, K] in `dtype` values (MLX rounding,
    round(round(scale * q) + bias)): every row gathered through the
    embedding restatement."""
    N = wq.shape[0]
    return quantized_embedding(np.arange(N, dtype=np.int32), wq, scales, biases, group, bits, dtype)


def logits_pick(logits, dtype="bfloat16"):
    x = _f32(logits).reshape(-1)
    t, lp, lse = C.c_int32(0), C.c_float(0), C.c_float(0)
    lib().orc_logits_pick(x, x.size, DT[dtype], C.byref(t), C.byref(lp), C.byref(lse))
    return int(t.value), float(lp.value), float(lse.value)


def linear(x, w, bias=None, act=0):
    x, w = _f32(x), _f32(w)
    K = x.shape[-1]
    M = x.size // K
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    lib().orc_linear(x.reshape(M, K), w, _opt(bias), y, M, N, K, act)
    return y.reshape(*x.shape[:-1], N)


def gelu_mlp(x, w1, b1, w2, b2):
    """Linear -> GELU -> Linear (examples/tiny_mlp.py:5-6 shape family)."""
    return linear(linear(x, w1, b1, act=1), w2, b2, act=0)


def erf(x: float) -> float:
    return float(lib().orc_erf(x))


def mamba_scan(x, dt_raw, dt_bias, A, B, Cm, D, z, h_state=None, dtype="float16"):
    x = _f32(x)
    L, d_inner = x.shape[-2], x.shape[-1]
    d_state = np.asarray(A).shape[-1]
    y = np.empty_like(x)
    hs = None if h_state is None else h_state
    lib().orc_mamba_scan(x, _f32(dt_raw), _opt(dt_bias), _f32(A), _f32(B), _f32(Cm), _opt(D), _f32(z), y,
                         None if hs is None else hs.ctypes.data_as(C.c_void_p), L, d_inner, d_state, DT[dtype])
    return y


def causal_conv1d(x, w, bias=None, state=None, silu=True, dtype="float16"):
    x = _f32(x)
    L, Cn = x.shape[-2], x.shape[-1]
    W = np.asarray(w).shape[-1]
    y = np.empty_like(x)
    lib().orc_causal_conv1d(x, _f32(w), _opt(bias), _opt(state), y, L, Cn, W, int(silu), DT[dtype])
    return y


def conv1d(x, w, bias=None, stride=1, padding=0, act=0, dtype="float16"):
    """mx.conv1d (channels-last x [N, L, Cin], w [Cout, K, Cin]) + bias + optional GELU
    (mlx-whisper's conv stem), each op rounded to dtype."""
    x, w = _f32(x), _f32(w)
    N, L, Cin = x.shape
    Cout, K, _ = w.shape
    Lout = (L + 2 * padding - K) // stride + 1
    y = np.empty((N, Lout, Cout), np.float32)
    lib().orc_conv1d(x, w, _opt(bias), y, N, L, Cin, Cout, K, stride, padding, act, DT[dtype])
    return y


def linear_lp(x, w, bias=None, act=0, dtype="float16"):
    """nn.Linear in a 16-bit dtype: round(x w^T + bias), then GELU (act=1) rounded."""
    x, w = _f32(x), _f32(w)
    K = x.shape[-1]
    M = x.size // K
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    lib().orc_linear_lp(x.reshape(M, K), w, _opt(bias), y, M, N, K, act, DT[dtype])
    return y.reshape(*x.shape[:-1], N)
