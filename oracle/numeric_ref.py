"""TEST INFRASTRUCTURE — numpy restatement of the reference's output contract.

Follows autotuner_runtime/numeric.py:50-107 (compare), :111-122 (check),
autotuner_runtime/exact.py:5-10 (bitwise_equal), autotuner/ladder/numeric.py:
22-35 (max_abs_diff) and autotuner/artifact/validate.py:79-100 (_cosine),
elementwise in float32 as MLX evaluates them. Pinned against the reference's
own known-answer cases (tests/golden/numeric_contract.json, transcribed from
tests/test_numeric_contract.py). Used only by tests/ as the checker of the
GPU diff reduction.
"""
from __future__ import annotations

import math

import numpy as np

MAX_TOLERANCE = float.fromhex("0x1.fffffep+127")
FLOAT_KINDS = ("float16", "bfloat16", "float32")


def validate_tolerances(values):
    if len(values) != 2 or any(isinstance(v, bool) or not math.isfinite(v) or v < 0 for v in values):
        raise ValueError("tolerances must be two finite non-negative numbers (rtol, atol)")
    if any(v > MAX_TOLERANCE for v in values):
        raise ValueError("tolerances must fit in float32, the comparison dtype")


def compare(c: np.ndarray, r: np.ndarray, rtol: float, atol: float, wobble: float = 0.0, *,
            floating: bool = True) -> dict:
    """Returns {passed, reason, max_excess, index, over}."""
    validate_tolerances((rtol, atol))
    if c.shape != r.shape:
        return dict(passed=False, reason="shape", max_excess=math.inf, index=None)
    if c.size == 0:
        return dict(passed=True, reason="", max_excess=0.0, index=None)
    if not floating:
        diff = c != r
        if diff.any():
            return dict(passed=False, reason="tolerance", max_excess=math.inf,
                        index=np.unravel_index(int(np.argmax(diff)), c.shape))
        return dict(passed=True, reason="", max_excess=0.0, index=None)
    c = c.astype(np.float32)
    r = r.astype(np.float32)
    with np.errstate(all="ignore"):
        ok = (np.isfinite(r) & np.isfinite(c)) | (np.isnan(r) & np.isnan(c)) | (np.isinf(r) & (c == r))
        if not ok.all():
            viol = ~ok
            return dict(passed=False, reason="nonfinite_pattern", max_excess=math.inf,
                        index=np.unravel_index(int(np.argmax(viol)), c.shape), violations=int(viol.sum()))
        f32 = np.float32
        allowed = np.maximum(f32(atol) + f32(rtol) * np.abs(r), f32(wobble))
        excess = np.where(np.isfinite(r), np.abs(c - r) - allowed, np.zeros_like(r))
        scale = np.maximum(np.maximum(np.abs(c), np.abs(r)), f32(1.0))
        scaled = np.abs(c / scale - r / scale) - (f32(atol) / scale + f32(rtol) * np.abs(r / scale))
        excess = np.where(np.isfinite(r) & np.isnan(excess), scaled * scale, excess)
    if np.isnan(excess).any():
        return dict(passed=False, reason="nonfinite_error", max_excess=None, index=None)
    worst = float(excess.max())
    index = np.unravel_index(int(np.argmax(excess)), c.shape)
    if worst > 0:
        return dict(passed=False, reason="tolerance", max_excess=worst, index=index,
                    over=int((excess > 0).sum()))
    return dict(passed=True, reason="", max_excess=worst, index=index, over=0)


def bitwise_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and a.tobytes() == b.tobytes()


def check(c, r, *, exact=True, rtol=0.0, atol=0.0, floating=True) -> dict:
    if not exact:
        return compare(c, r, rtol, atol, floating=floating)
    if c.shape != r.shape:
        return dict(passed=False, reason="shape", max_excess=None)
    if not bitwise_equal(c, r):
        return dict(passed=False, reason="exact", max_excess=None)
    return dict(passed=True, reason="", max_excess=0.0)


def max_abs_diff(a: np.ndarray, b: np.ndarray, floating=True) -> float:
    if a.shape != b.shape:
        return math.inf
    if a.size == 0:
        return 0.0
    if not floating:
        return 0.0 if np.array_equal(a, b) else math.inf
    af, bf = a.astype(np.float32), b.astype(np.float32)
    with np.errstate(all="ignore"):
        ok = (np.isfinite(bf) & np.isfinite(af)) | (np.isnan(bf) & np.isnan(af)) | (np.isinf(bf) & (af == bf))
        if not ok.all():
            return math.inf
        return float(np.where(np.isfinite(bf), np.abs(af - bf), 0).max())


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    """validate.py `_cosine` for one tensor pair."""
    xf = np.where(np.isfinite(a), a, 0).astype(np.float32).reshape(-1)
    yf = np.where(np.isfinite(b), b, 0).astype(np.float32).reshape(-1)
    if xf.size == 0:
        return 1.0
    sx, sy = float(np.abs(xf).max()), float(np.abs(yf).max())
    if sx == 0.0 or sy == 0.0:
        return 1.0 if sx == sy else 0.0
    xf, yf = xf / np.float32(sx), yf / np.float32(sy)
    denom = math.sqrt(float(np.sum(xf * xf, dtype=np.float64)) * float(np.sum(yf * yf, dtype=np.float64)))
    c = float(np.sum(xf * yf, dtype=np.float64)) / denom
    if not math.isfinite(c):
        return -1.0
    return max(-1.0, min(1.0, c))
