"""ctypes binding of libmt.so — the C ABI declared in include/mt.h.

Every wrapper takes torch tensors that already live on the current CUDA
device, passes their data pointers and the current torch stream, and raises
MTError with the library's message when an entry point returns non-zero.
There is no fallback: if libmt.so is missing or the device is not a CUDA
device, the call raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmt.so"

# element-type codes of include/mt.h
MT_BF16, MT_F16, MT_F32, MT_I32, MT_U32, MT_I64, MT_U8, MT_BOOL, MT_I8, MT_I16, MT_U16, MT_U64 = range(12)

_DTYPE_CODES = {
    torch.bfloat16: MT_BF16, torch.float16: MT_F16, torch.float32: MT_F32,
    torch.int32: MT_I32, torch.uint32: MT_U32, torch.int64: MT_I64, torch.uint8: MT_U8,
    torch.bool: MT_BOOL, torch.int8: MT_I8, torch.int16: MT_I16, torch.uint16: MT_U16,
    torch.uint64: MT_U64,
}

ERRORS = {-1: "invalid argument", -2: "unsupported", -3: "workspace", -4: "cuda", -5: "device timeout"}


class MTError(RuntimeError):
    """A libmt entry point returned an error code."""

    def __init__(self, code: int, symbol: str, message: str):
        super().__init__(f"{symbol}: {ERRORS.get(code, code)}: {message}")
        self.code = code
        self.symbol = symbol


class DiffStats(C.Structure):
    """Mirror of mt_diff_stats."""
    _fields_ = [
        ("max_excess", C.c_double), ("max_abs", C.c_double),
        ("dot_ab", C.c_double), ("dot_aa", C.c_double), ("dot_bb", C.c_double),
        ("amax_a", C.c_double), ("amax_b", C.c_double),
        ("excess_index", C.c_int64), ("over_count", C.c_int64),
        ("nonfinite_violations", C.c_int64), ("first_violation", C.c_int64),
        ("bit_mismatches", C.c_int64), ("first_mismatch", C.c_int64),
        ("nan_excess", C.c_int64),
    ]


P, I64, I32, F32, SZ = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# symbol -> (restype, argtypes), in include/mt.h order
SIGNATURES = {
    "mt_version": (C.c_int, []),
    "mt_kernel_launches": (C.c_uint64, []),
    "mt_last_error_string": (C.c_char_p, []),
    "mt_device_status": (C.c_int, [C.POINTER(C.c_int), I32]),
    "mt_sm_count": (C.c_int, [C.POINTER(C.c_int)]),
    "mt_quantized_matmul": (C.c_int, [P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, SZ, P]),
    "mt_quantized_matmul_residual": (C.c_int, [P, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, SZ, P]),
    "mt_quantized_matmul_residual_rms_norm": (
        C.c_int, [P, P, P, P, P, P, F32, P, P, I64, I64, I64, I32, I32, I32, P, SZ, P]),
    "mt_quantized_matmul_swiglu": (C.c_int, [P, P, P, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, SZ, P]),
    "mt_quantized_matmul_multi": (
        C.c_int, [P, P, P, P, P, I64, P, P, P, P, I64, P, P, P, P, I64, I64, I64, I32, I32, I32, P, SZ, P]),
    "mt_rms_norm_quantized_matmul_multi": (
        C.c_int, [P, P, F32, P, P, P, P, I64, P, P, P, P, I64, P, P, P, P, I64, I64, I64, I32, I32, I32, P]),
    "mt_rms_norm_quantized_matmul_swiglu": (
        C.c_int, [P, P, F32, P, P, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P]),
    "mt_qk_norm_rope_sdpa_decode": (
        C.c_int, [P, P, P, I64, I64, P, P, F32, P, P, P, I64, I64, I64, I64, I64, I64, F32, F32, I32, P]),
    "mt_conv1d": (C.c_int, [P, P, P, P, I64, I64, I64, I64, I32, I32, I32, I32, I32, P]),
    "mt_qmm_workspace_bytes": (C.c_size_t, [I64, I64, I64, I32, I32]),
    "mt_qmm_partition_check": (C.c_int, [I64, I32, I32, I32, P]),
    "mt_rms_norm": (C.c_int, [P, P, F32, P, I64, I64, I32, P]),
    "mt_add_rms_norm": (C.c_int, [P, P, P, F32, P, P, I64, I64, I32, P]),
    "mt_rope": (C.c_int, [P, P, I64, I64, I64, I64, I32, I32, F32, F32, I64, I32, P]),
    "mt_rope_strided": (C.c_int, [P, P, I64, I64, I64, I64, I32, I32, F32, F32, I64, I64, I64, I64, I64, I64, I64,
                                  I32, P]),
    "mt_qk_norm_rope_cache": (
        C.c_int, [P, P, P, I64, I64, P, P, F32, P, P, P, I64, I64, I64, I64, I64, I64, F32, I32, P]),
    "mt_swiglu": (C.c_int, [P, P, P, I64, I32, P]),
    "mt_sdpa": (C.c_int, [P, P, P, P, I64, I64, I64, I64, I64, I64, F32, I32, I64,
                          I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I32, P]),
    "mt_quantized_embedding": (C.c_int, [P, P, P, P, P, I64, I64, I64, I32, I32, I32, P]),
    "mt_logits_pick": (C.c_int, [P, I64, I32, P, P, P, P]),
    "mt_diff_workspace_bytes": (C.c_size_t, [I64]),
    "mt_diff_reduce": (C.c_int, [P, P, I64, I32, F32, F32, F32, P, P, SZ, P]),
    "mt_diff_reduce_noalloc": (C.c_int, [P, P, I64, I32, F32, F32, F32, P, P]),
    "mt_add": (C.c_int, [P, P, P, I64, I64, I32, P]),
    "mt_embedding": (C.c_int, [P, P, P, I64, I64, I64, I32, P]),
    "mt_linear": (C.c_int, [P, P, P, P, I64, I64, I64, I32, I32, P]),
    "mt_linear_residual": (C.c_int, [P, P, P, P, P, I64, I64, I64, I32, P]),
    "mt_layer_norm": (C.c_int, [P, P, P, F32, P, I64, I64, I32, P]),
    "mt_mamba_scan": (C.c_int, [P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I32, P]),
    "mt_causal_conv1d": (C.c_int, [P, P, P, P, P, I64, I64, I32, I32, I32, P]),
}

_lib = None
_lock = threading.Lock()
CALLS = [0]  # entry-point calls made through this binding (each is one or more kernel launches)


def load(path: str | Path | None = None) -> C.CDLL:
    """Load libmt.so once (raises FileNotFoundError if it was never built)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise FileNotFoundError(
                f"{p} is missing: build it with `python -m metal_autotune_b200.build` "
                "(the region kernels have no fallback)")
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def kernel_launches() -> int:
    """Kernels libmt has launched in this process (host-side count; a launch
    captured into a CUDA graph counts once)."""
    return int(load().mt_kernel_launches())


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dt]
    except KeyError:
        raise TypeError(f"dtype {dt} has no libmt code") from None


def _check(rc: int, symbol: str) -> None:
    if rc != 0:
        msg = load().mt_last_error_string()
        raise MTError(rc, symbol, msg.decode() if msg else "")


def call(symbol: str, *args) -> int:
    """Call an int-returning entry point and raise on a non-zero code."""
    rc = getattr(load(), symbol)(*args)
    CALLS[0] += 1
    _check(rc, symbol)
    return rc


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libmt kernels take CUDA tensors; got a tensor on " + str(t.device))
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dense(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be row-contiguous")
    return t


# ------------------------------------------------------------------ workspace
class Workspace:
    """Per-device scratch buffer for kernels that split work (qmm split-K,
    diff reduction). Allocated once, zero-filled, grown on demand; every
    kernel that uses it leaves its counters zeroed. Use from one stream."""

    _per_device: dict[int, "Workspace"] = {}

    def __init__(self, device: int, nbytes: int):
        self.device = device
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=f"cuda:{device}")

    @classmethod
    def get(cls, nbytes: int, device: int | None = None) -> "Workspace":
        dev = torch.cuda.current_device() if device is None else device
        ws = cls._per_device.get(dev)
        if ws is None or ws.buf.numel() < nbytes:
            size = max(nbytes, 64 << 20, 0 if ws is None else ws.buf.numel())
            ws = cls(dev, size)
            cls._per_device[dev] = ws
        return ws

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    def reset(self) -> None:
        """Re-zero after an aborted kernel may have left counters non-zero."""
        self.buf.zero_()


def qmm_workspace_bytes(M: int, n_total: int, K: int, bits: int, kind: int = 0) -> int:
    return int(load().mt_qmm_workspace_bytes(M, n_total, K, bits, kind))


# ------------------------------------------------------------------ wrappers
def _qmm_common(x: torch.Tensor, w: torch.Tensor, group_size: int, bits: int):
    _dense(x, "x")
    _dense(w, "w")
    if w.dtype not in (torch.int32, torch.uint32):
        raise TypeError("packed weights must be uint32 (or int32 bit patterns)")
    K = x.shape[-1]
    M = x.numel() // K if K else 0
    N = w.shape[0]
    if w.shape[1] * (32 // bits) != K:
        raise ValueError(f"w {tuple(w.shape)} does not pack K={K} at {bits} bits")
    return M, N, K


def quantized_matmul(x, w, scales, biases, *, group_size=64, bits=4, out=None, residual=None):
    """mx.quantized_matmul(x, w, scales, biases, transpose=True, group_size, bits), optionally
    fused with `+ residual`."""
    M, N, K = _qmm_common(x, w, group_size, bits)
    y = out if out is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    ws = Workspace.get(qmm_workspace_bytes(M, N, K, bits, 0))
    if residual is None:
        call("mt_quantized_matmul", _ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(y), M, N, K,
             group_size, bits, dtype_code(x.dtype), ws.ptr, ws.nbytes, _stream())
    else:
        _dense(residual, "residual")
        call("mt_quantized_matmul_residual", _ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(residual),
             _ptr(y), M, N, K, group_size, bits, dtype_code(x.dtype), ws.ptr, ws.nbytes, _stream())
    return y


def quantized_matmul_residual_rms_norm(x, w, scales, biases, residual, norm_w, eps, *, group_size=64, bits=4,
                                       h=None, y=None):
    M, N, K = _qmm_common(x, w, group_size, bits)
    shape = (*x.shape[:-1], N)
    h = h if h is not None else torch.empty(shape, dtype=x.dtype, device=x.device)
    y = y if y is not None else torch.empty(shape, dtype=x.dtype, device=x.device)
    ws = Workspace.get(qmm_workspace_bytes(M, N, K, bits, 0))
    call("mt_quantized_matmul_residual_rms_norm", _ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(residual),
         _ptr(norm_w), float(eps), _ptr(h), _ptr(y), M, N, K, group_size, bits, dtype_code(x.dtype), ws.ptr,
         ws.nbytes, _stream())
    return h, y


def quantized_matmul_swiglu(x, wg, sg, bg, wu, su, bu, *, group_size=64, bits=4, out=None):
    M, N, K = _qmm_common(x, wg, group_size, bits)
    y = out if out is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    ws = Workspace.get(qmm_workspace_bytes(M, 2 * N, K, bits, 1))
    call("mt_quantized_matmul_swiglu", _ptr(x), _ptr(wg), _ptr(sg), _ptr(bg), _ptr(wu), _ptr(su), _ptr(bu),
         _ptr(y), M, N, K, group_size, bits, dtype_code(x.dtype), ws.ptr, ws.nbytes, _stream())
    return y


def quantized_matmul_multi(x, sets, *, group_size=64, bits=4, outs=None):
    """sets: up to three (w, scales, biases) triples sharing x; returns their outputs."""
    if not 1 <= len(sets) <= 3:
        raise ValueError("one to three weight sets")
    M, _, K = _qmm_common(x, sets[0][0], group_size, bits)
    ys = []
    args = []
    for i in range(3):
        if i < len(sets):
            w, s, b = sets[i]
            N = w.shape[0]
            y = outs[i] if outs is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
            ys.append(y)
            args += [_ptr(w), _ptr(s), _ptr(b), _ptr(y), N]
        else:
            args += [None, None, None, None, 0]
    n_total = sum(w.shape[0] for w, _, _ in sets)
    ws = Workspace.get(qmm_workspace_bytes(M, n_total, K, bits, 0))
    call("mt_quantized_matmul_multi", _ptr(x), *args, M, K, group_size, bits, dtype_code(x.dtype), ws.ptr,
         ws.nbytes, _stream())
    return ys


def rms_norm_quantized_matmul_multi(x, norm_w, eps, sets, *, group_size=64, bits=4, outs=None):
    """Decode (M <= 4): quantized_matmul_multi(rms_norm(x, norm_w, eps), sets) in one launch."""
    if not 1 <= len(sets) <= 3:
        raise ValueError("one to three weight sets")
    M, _, K = _qmm_common(x, sets[0][0], group_size, bits)
    _dense(norm_w, "norm_w")
    ys = []
    args = []
    for i in range(3):
        if i < len(sets):
            w, s, b = sets[i]
            N = w.shape[0]
            y = outs[i] if outs is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
            ys.append(y)
            args += [_ptr(w), _ptr(s), _ptr(b), _ptr(y), N]
        else:
            args += [None, None, None, None, 0]
    call("mt_rms_norm_quantized_matmul_multi", _ptr(x), _ptr(norm_w), float(eps), *args, M, K, group_size, bits,
         dtype_code(x.dtype), _stream())
    return ys


def rms_norm_quantized_matmul_swiglu(x, norm_w, eps, wg, sg, bg, wu, su, bu, *, group_size=64, bits=4, out=None):
    """Decode (M <= 4): quantized_matmul_swiglu(rms_norm(x, norm_w, eps), ...) in one launch."""
    M, N, K = _qmm_common(x, wg, group_size, bits)
    _dense(norm_w, "norm_w")
    y = out if out is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    call("mt_rms_norm_quantized_matmul_swiglu", _ptr(x), _ptr(norm_w), float(eps), _ptr(wg), _ptr(sg), _ptr(bg),
         _ptr(wu), _ptr(su), _ptr(bu), _ptr(y), M, N, K, group_size, bits, dtype_code(x.dtype), _stream())
    return y


def rms_norm(x, w, eps, *, out=None):
    _dense(x, "x")
    y = out if out is not None else torch.empty_like(x)
    D = x.shape[-1]
    call("mt_rms_norm", _ptr(x), _ptr(w), float(eps), _ptr(y), x.numel() // D, D, dtype_code(x.dtype), _stream())
    return y


def add_rms_norm(x, residual, w, eps, *, h=None, y=None):
    _dense(x, "x")
    _dense(residual, "residual")
    h = h if h is not None else torch.empty_like(x)
    y = y if y is not None else torch.empty_like(x)
    D = x.shape[-1]
    call("mt_add_rms_norm", _ptr(x), _ptr(residual), _ptr(w), float(eps), _ptr(h), _ptr(y), x.numel() // D, D,
         dtype_code(x.dtype), _stream())
    return h, y


def layer_norm(x, w, b, eps, *, out=None):
    _dense(x, "x")
    y = out if out is not None else torch.empty_like(x)
    D = x.shape[-1]
    call("mt_layer_norm", _ptr(x), _ptr(w), _ptr(b), float(eps), _ptr(y), x.numel() // D, D, dtype_code(x.dtype),
         _stream())
    return y


def rope(x, dims, *, traditional=False, base=10000.0, scale=1.0, offset=0, out=None):
    """mx.fast.rope over x [..., L, D] (position along axis -2)."""
    _dense(x, "x")
    y = out if out is not None else torch.empty_like(x)
    L, D = x.shape[-2], x.shape[-1]
    lead = x.numel() // (L * D) if L * D else 0
    call("mt_rope", _ptr(x), _ptr(y), 1, lead, L, D, int(dims), int(bool(traditional)), float(base), float(scale),
         int(offset), dtype_code(x.dtype), _stream())
    return y


def rope_bhld(x, dims, *, traditional=False, base=10000.0, scale=1.0, offset=0, out=None):
    """mx.fast.rope over a 4-D view x [B, H, L, D] of any strides (D contiguous), e.g. the
    transposed [B, L, H, D] projection output; out is a dense [B, H, L, D] by default."""
    if x.dim() != 4 or x.stride(3) != 1:
        raise ValueError("x must be a 4-D view [B, H, L, D] with D contiguous")
    B, H, L, D = x.shape
    y = out if out is not None else torch.empty((B, H, L, D), dtype=x.dtype, device=x.device)
    if y.shape != x.shape or y.stride(3) != 1:
        raise ValueError("out must have x's shape with D contiguous")
    call("mt_rope_strided", _ptr(x), _ptr(y), B, H, L, D, int(dims), int(bool(traditional)), float(base),
         float(scale), int(offset), x.stride(0), x.stride(1), x.stride(2), y.stride(0), y.stride(1), y.stride(2),
         dtype_code(x.dtype), _stream())
    return y


def qk_norm_rope_cache(q, k, v, q_norm_w, k_norm_w, eps, q_out, k_cache, v_cache, *, n_heads, n_kv_heads,
                       offset, rope_base, head_dim=128):
    """q [T, Hq*D], k/v [T, Hkv*D] rows (any row stride) -> q_out [Hq, T, D], caches [Hkv, cap, D]."""
    T = q.shape[0]
    call("mt_qk_norm_rope_cache", _ptr(q), _ptr(k), _ptr(v), q.stride(0), k.stride(0), _ptr(q_norm_w),
         _ptr(k_norm_w), float(eps), _ptr(q_out), _ptr(k_cache), _ptr(v_cache), T, n_heads, n_kv_heads, head_dim,
         k_cache.shape[-2], int(offset), float(rope_base), dtype_code(q.dtype), _stream())


def qk_norm_rope_sdpa_decode(q, k, v, q_norm_w, k_norm_w, eps, k_cache, v_cache, *, n_heads, n_kv_heads, offset,
                             rope_base, scale, head_dim=128, out=None):
    """Decode: qk_norm_rope_cache + causal GQA attention in one launch. q [T, Hq*D], k/v [T, Hkv*D]
    rows; caches [Hkv, cap, D] get the new rows; returns o [T, Hq*D]."""
    T = q.shape[0]
    o = out if out is not None else torch.empty(T, n_heads * head_dim, dtype=q.dtype, device=q.device)
    call("mt_qk_norm_rope_sdpa_decode", _ptr(q), _ptr(k), _ptr(v), q.stride(0), k.stride(0), _ptr(q_norm_w),
         _ptr(k_norm_w), float(eps), _ptr(o), _ptr(k_cache), _ptr(v_cache), T, n_heads, n_kv_heads, head_dim,
         k_cache.shape[-2], int(offset), float(rope_base), float(scale), dtype_code(q.dtype), _stream())
    return o


def conv1d(x, w, bias=None, *, stride=1, padding=0, act=0, out=None):
    """mx.conv1d (channels-last x [N, L, Cin], w [Cout, K, Cin]) + optional bias and GELU (act=1)."""
    _dense(x, "x")
    _dense(w, "w")
    N, L, Cin = x.shape
    Cout, K, _ = w.shape
    Lout = (L + 2 * padding - K) // stride + 1
    y = out if out is not None else torch.empty(N, Lout, Cout, dtype=x.dtype, device=x.device)
    call("mt_conv1d", _ptr(x), _ptr(w), _ptr(bias) if bias is not None else None, _ptr(y), N, L, Cin, Cout, K,
         stride, padding, act, dtype_code(x.dtype), _stream())
    return y


def swiglu(gate, up, *, out=None):
    _dense(gate, "gate")
    _dense(up, "up")
    y = out if out is not None else torch.empty_like(gate)
    call("mt_swiglu", _ptr(gate), _ptr(up), _ptr(y), gate.numel(), dtype_code(gate.dtype), _stream())
    return y


def sdpa(q, k, v, *, scale, causal, q_offset=0, out=None, out_layout="bhld"):
    """q [B, Hq, Lq, D], k/v [B, Hkv, Lk, D] (any strides with D contiguous).
    out_layout 'bhld' -> [B, Hq, Lq, D]; 'blhd' -> [B, Lq, Hq, D] (heads concatenated per token)."""
    B, Hq, Lq, D = q.shape
    Hkv, Lk = k.shape[1], k.shape[2]
    if out is None:
        shape = (B, Hq, Lq, D) if out_layout == "bhld" else (B, Lq, Hq, D)
        out = torch.empty(shape, dtype=q.dtype, device=q.device)
    if out_layout == "bhld":
        os_b, os_h, os_l = out.stride(0), out.stride(1), out.stride(2)
    else:
        os_b, os_h, os_l = out.stride(0), out.stride(2), out.stride(1)
    call("mt_sdpa", _ptr(q), _ptr(k), _ptr(v), _ptr(out), B, Hq, Hkv, Lq, Lk, D, float(scale), int(bool(causal)),
         int(q_offset), q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0),
         v.stride(1), v.stride(2), os_b, os_h, os_l, dtype_code(q.dtype), _stream())
    return out


def add(x, r, *, out=None):
    """round(x + r) with r repeated over x's leading elements (r.numel() divides x.numel())."""
    _dense(x, "x")
    _dense(r, "r")
    y = out if out is not None else torch.empty_like(x)
    call("mt_add", _ptr(x), _ptr(r), _ptr(y), x.numel(), r.numel(), dtype_code(x.dtype), _stream())
    return y


def embedding(tokens, table, *, out=None):
    """table[tokens] for a dense [vocab, D] table."""
    _dense(table, "table")
    T = tokens.numel()
    D = table.shape[1]
    y = out if out is not None else torch.empty(*tokens.shape, D, dtype=table.dtype, device=table.device)
    call("mt_embedding", _ptr(tokens), _ptr(table), _ptr(y), T, table.shape[0], D, dtype_code(table.dtype),
         _stream())
    return y


def quantized_embedding(tokens, w, scales, biases, *, group_size=64, bits=4, dtype=None, out=None):
    T = tokens.numel()
    D = w.shape[1] * (32 // bits)
    dt = dtype or scales.dtype
    y = out if out is not None else torch.empty(*tokens.shape, D, dtype=dt, device=w.device)
    call("mt_quantized_embedding", _ptr(tokens), _ptr(w), _ptr(scales), _ptr(biases), _ptr(y), T, w.shape[0], D,
         group_size, bits, dtype_code(dt), _stream())
    return y


def logits_pick(logits, *, token=None, logprob=None, lse=None):
    """Greedy token, its log-probability and logsumexp of one row of logits."""
    n = logits.numel()
    dev = logits.device
    token = token if token is not None else torch.empty(1, dtype=torch.int32, device=dev)
    logprob = logprob if logprob is not None else torch.empty(1, dtype=torch.float32, device=dev)
    lse = lse if lse is not None else torch.empty(1, dtype=torch.float32, device=dev)
    call("mt_logits_pick", _ptr(logits), n, dtype_code(logits.dtype), _ptr(token), _ptr(logprob), _ptr(lse),
         _stream())
    return token, logprob, lse


def diff_reduce(a, b, *, rtol=0.0, atol=0.0, wobble=0.0, stats=None):
    """One-pass comparison statistics of candidate a vs reference b (device struct in `stats`, a
    uint8 tensor of sizeof(DiffStats) bytes). Returns the stats tensor."""
    if a.shape != b.shape or a.dtype != b.dtype:
        raise ValueError("diff_reduce compares tensors of one shape and dtype")
    a = a.contiguous()
    b = b.contiguous()
    n = a.numel()
    if stats is None:
        stats = torch.zeros(C.sizeof(DiffStats), dtype=torch.uint8, device=a.device)
    need = int(load().mt_diff_workspace_bytes(n))
    ws = Workspace.get(need)
    call("mt_diff_reduce", _ptr(a) if n else None, _ptr(b) if n else None, n, dtype_code(a.dtype), float(rtol),
         float(atol), float(wobble), _ptr(stats), ws.ptr, ws.nbytes, _stream())
    return stats


def read_diff_stats(stats: torch.Tensor) -> DiffStats:
    raw = bytes(stats.cpu().numpy().tobytes())
    return DiffStats.from_buffer_copy(raw)


def linear(x, w, bias=None, *, act=0, out=None):
    _dense(x, "x")
    _dense(w, "w")
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0]
    y = out if out is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    call("mt_linear", _ptr(x), _ptr(w), _ptr(bias), _ptr(y), M, N, K, int(act), dtype_code(x.dtype), _stream())
    return y


def linear_residual(x, w, bias, residual, *, out=None):
    """round(round(x @ w.T + bias) + residual) in x's 16-bit dtype (tcgen05 GEMM)."""
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0]
    _dense(x, "x")
    _dense(w, "w")
    _dense(residual, "residual")
    y = out if out is not None else torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    call("mt_linear_residual", _ptr(x), _ptr(w), _ptr(bias) if bias is not None else None, _ptr(residual), _ptr(y),
         M, N, K, dtype_code(x.dtype), _stream())
    return y


def mamba_scan(x, dt_raw, dt_bias, A, B, Cm, D, z, *, h_state=None, out=None):
    L, d_inner = x.shape[-2], x.shape[-1]
    d_state = A.shape[-1]
    y = out if out is not None else torch.empty_like(x)
    call("mt_mamba_scan", _ptr(x), _ptr(dt_raw), _ptr(dt_bias), _ptr(A), _ptr(B), _ptr(Cm), _ptr(D), _ptr(z),
         _ptr(y), _ptr(h_state), L, d_inner, d_state, dtype_code(x.dtype), _stream())
    return y


def causal_conv1d(x, weight, bias=None, *, conv_state=None, silu=True, out=None):
    L, Cn = x.shape[-2], x.shape[-1]
    width = weight.shape[-1]
    y = out if out is not None else torch.empty_like(x)
    call("mt_causal_conv1d", _ptr(x), _ptr(weight), _ptr(bias), _ptr(conv_state), _ptr(y), L, Cn, width,
         int(bool(silu)), dtype_code(x.dtype), _stream())
    return y


def device_status(clear: bool = True) -> int:
    v = C.c_int(0)
    call("mt_device_status", C.byref(v), int(clear))
    return v.value


def sm_count() -> int:
    v = C.c_int(0)
    call("mt_sm_count", C.byref(v))
    return v.value


def version() -> tuple[int, int, int]:
    v = load().mt_version()
    return (v >> 16, (v >> 8) & 0xFF, v & 0xFF)
