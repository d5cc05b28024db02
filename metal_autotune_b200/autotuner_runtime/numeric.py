"""Output contract shared by verification and exported bundles (the
reference's autotuner_runtime/numeric.py:1-137), evaluated on the GPU.

compare() runs one pass of the output-diff reduction kernel
(mt_diff_reduce) over candidate and reference and reads back one small
struct; the decision logic below is the reference's, in the same order:
shape, dtype, empty, exact match for non-floating outputs, the non-finite
pattern rule, then |c - r| <= max(atol + rtol*|r|, wobble) with the
overflow-safe scaled excess. Tensors must live on a CUDA device (CPU tensors
are moved there; without a GPU these functions raise).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from types import MappingProxyType

import torch

from .. import lib as _mt

FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)
MAX_TOLERANCE = float.fromhex("0x1.fffffep+127")  # largest finite float32
DEFAULT_TOLERANCES = MappingProxyType({
    "float32": (1e-5, 1e-6),
    "float16": (1e-2, 2e-2),
    "bfloat16": (2e-2, 4e-2),
})


def validate_tolerances(values) -> None:
    if len(values) != 2 or any(isinstance(v, bool) or not math.isfinite(v) or v < 0 for v in values):
        raise ValueError("tolerances must be two finite non-negative numbers (rtol, atol)")
    if any(v > MAX_TOLERANCE for v in values):
        raise ValueError("tolerances must fit in float32, the comparison dtype")


def tolerance_for(dtype, override=None) -> tuple[float, float]:
    name = str(dtype).removeprefix("torch.")
    if override is not None:
        validate_tolerances(override)
        return tuple(override)
    return DEFAULT_TOLERANCES.get(name, (0.0, 0.0))


@dataclass(frozen=True)
class CompareResult:
    passed: bool
    reason: str                      # "" | shape | dtype | nonfinite_pattern | nonfinite_error | tolerance | exact
    max_excess: float | None
    index: tuple[int, ...] | None
    detail: str = ""


def _cuda(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t
    if not torch.cuda.is_available():
        raise RuntimeError("the output-diff reduction runs on a CUDA device; none is available")
    return t.cuda()


def _unravel(flat: int, shape: tuple[int, ...]) -> tuple[int, ...]:
    idx = []
    for dim in reversed(shape):
        flat, r = divmod(flat, dim)
        idx.append(r)
    return tuple(reversed(idx))


def diff_stats(candidate: torch.Tensor, reference: torch.Tensor, rtol: float = 0.0, atol: float = 0.0,
               wobble: float = 0.0) -> _mt.DiffStats:
    """One GPU pass; returns the host copy of mt_diff_stats."""
    c, r = _cuda(candidate), _cuda(reference)
    with torch.cuda.device(c.device):
        stats = _mt.diff_reduce(c, r, rtol=rtol, atol=atol, wobble=wobble)
        return _mt.read_diff_stats(stats)


def compare(candidate: torch.Tensor, reference: torch.Tensor, rtol: float, atol: float,
            wobble_floor: float = 0.0) -> CompareResult:
    validate_tolerances((rtol, atol))
    if tuple(candidate.shape) != tuple(reference.shape):
        return CompareResult(False, "shape", float("inf"), None,
                             f"{tuple(candidate.shape)} != {tuple(reference.shape)}")
    if candidate.dtype != reference.dtype:
        return CompareResult(False, "dtype", float("inf"), None, f"{candidate.dtype} != {reference.dtype}")
    if candidate.numel() == 0:
        return CompareResult(True, "", 0.0, None)
    shape = tuple(reference.shape)
    s = diff_stats(candidate, reference, rtol, atol, wobble_floor)
    if reference.dtype not in FLOAT_DTYPES:
        # indices, masks and packed words are exact values
        if s.bit_mismatches:
            return CompareResult(False, "tolerance", float("inf"), _unravel(s.first_mismatch, shape),
                                 "non-floating outputs must match exactly")
        return CompareResult(True, "", 0.0, None)
    if s.nonfinite_violations:
        return CompareResult(False, "nonfinite_pattern", float("inf"), _unravel(s.first_violation, shape),
                             f"{s.nonfinite_violations} elements break the non-finite pattern")
    if s.nan_excess:
        return CompareResult(False, "nonfinite_error", None, None, "comparison produced a NaN error")
    worst = float(s.max_excess)
    index = _unravel(s.excess_index, shape)
    if worst > 0:
        return CompareResult(False, "tolerance", worst, index, f"{s.over_count} elements over tolerance")
    return CompareResult(True, "", worst, index)


def check(candidate, reference, *, exact=True, rtol=0.0, atol=0.0) -> CompareResult:
    """Exact by default; tolerance is opt-in for floating evaluation changes (numeric.py:111-122)."""
    if not exact:
        return compare(candidate, reference, rtol, atol)
    if tuple(candidate.shape) != tuple(reference.shape):
        return CompareResult(False, "shape", None, None, "output shape changed")
    if candidate.dtype != reference.dtype:
        return CompareResult(False, "dtype", None, None, "output dtype changed")
    from .exact import bitwise_equal
    if not bitwise_equal(candidate, reference):
        return CompareResult(False, "exact", None, None, "output must match the original bit-for-bit")
    return CompareResult(True, "", 0.0, None)


def nonfinite_pattern_ok(candidate: torch.Tensor, reference: torch.Tensor) -> bool:
    """True when the candidate is finite where the reference is, NaN where NaN, same-signed inf where inf."""
    return diff_stats(candidate, reference).nonfinite_violations == 0


def max_abs_diff(a: torch.Tensor, b: torch.Tensor) -> float:
    """The run-to-run wobble (autotuner/ladder/numeric.py:22-35): worst |a-b|,
    0 where both share a non-finite pattern, inf when patterns differ."""
    if tuple(a.shape) != tuple(b.shape) or a.dtype != b.dtype:
        return float("inf")
    if a.numel() == 0:
        return 0.0
    s = diff_stats(a, b)
    if a.dtype not in FLOAT_DTYPES:
        return 0.0 if s.bit_mismatches == 0 else float("inf")
    if s.nonfinite_violations:
        return float("inf")
    return float(s.max_abs)


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    """Whole-output cosine of one tensor pair (autotuner/artifact/validate.py:79-100),
    non-finite values taken as 0, fp64 sums."""
    if tuple(a.shape) != tuple(b.shape) or a.dtype != b.dtype:
        return -1.0
    if a.numel() == 0:
        return 1.0
    s = diff_stats(a, b)
    if s.amax_a == 0.0 or s.amax_b == 0.0:
        return 1.0 if s.amax_a == s.amax_b else 0.0
    denom = math.sqrt(s.dot_aa * s.dot_bb)
    c = s.dot_ab / denom if denom > 0 else float("nan")
    if not math.isfinite(c):
        return -1.0
    return max(-1.0, min(1.0, c))
