"""Statistics of a paired timing comparison over CUDA-event samples.

Input: two aligned arrays of device milliseconds, one observation per
baseline/candidate pair (the timing harness pairs them in ABBA blocks, so
slow drift of the machine cancels within a pair). Everything is computed
with numpy from those arrays:

  delta_i = baseline_i - candidate_i   (positive: the candidate is faster)
  ratio_i = candidate_i / baseline_i   (pairs with a positive baseline)

The decision rule is the reference's contract (autotuner_runtime/stats.py:
12-15, 31-35): a median delta counts as a win (loss) only when it exceeds
max(margin, 3 * SE), where SE is the standard error of a median of normal
noise, 1.2533 * stdev(delta) / sqrt(n). The per-pair ratios give the
drift-immune summary: their median, and an agreement score
median / (median + interquartile range) in (0, 1], reported from four pairs
up (stats.py:66-81; quartiles by the exclusive rule, which is numpy's
"weibull" plotting position). A comparison whose numbers are not all finite,
or whose arrays disagree in length, never wins (stats.py:38-63).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Mapping, Sequence

import numpy as np

MEDIAN_SE_FACTOR = 1.2533  # SE of the median of normal noise, in sigma / sqrt(n)
MIN_PAIRS_FOR_AGREEMENT = 4


def decision(median_delta_ms: float, se_ms: float, margin_ms: float) -> int:
    """+1: resolved win, -1: resolved loss, 0: unresolved (or not a number)."""
    bar = max(margin_ms, 3.0 * se_ms)
    if median_delta_ms > bar:
        return 1
    if -median_delta_ms > bar:
        return -1
    return 0


@dataclass(frozen=True)
class PairedComparison:
    """Aligned samples and the statistics derived from them (milliseconds).

    Build it with `comparison_from_samples`; the derived fields are filled in
    from the two sample arrays and are not meant to be passed by hand."""
    baseline_ms: tuple[float, ...]
    candidate_ms: tuple[float, ...]
    deltas_ms: tuple[float, ...] = field(default=())
    median_baseline_ms: float = float("nan")
    median_delta_ms: float = float("nan")
    spread_ms: float = float("nan")     # sample stdev of the deltas (inf for one pair)
    sigma_ms: float = float("nan")      # standard error of the median delta
    n: int = 0
    ratios: tuple[float, ...] = ()
    median_ratio: float = 0.0
    stability: float = 0.0             # the agreement score, 0 below four pairs

    def wins_by(self, margin_ms: float) -> bool:
        return decision(self.median_delta_ms, self.sigma_ms, margin_ms) > 0

    def loses_by(self, margin_ms: float) -> bool:
        return decision(self.median_delta_ms, self.sigma_ms, margin_ms) < 0

    def well_formed(self) -> bool:
        """Every array has n entries and every number is finite."""
        if self.n < 1 or {len(self.baseline_ms), len(self.candidate_ms), len(self.deltas_ms)} != {self.n}:
            return False
        scalars = [self.median_baseline_ms, self.median_delta_ms, self.spread_ms, self.sigma_ms,
                   self.median_ratio, self.stability]
        arrays = np.concatenate([np.asarray(a, np.float64) for a in
                                 (self.baseline_ms, self.candidate_ms, self.deltas_ms, self.ratios, scalars)])
        return bool(np.isfinite(arrays).all())

    def as_record(self) -> dict:
        """Plain-dict form for JSON logs."""
        return {k: (list(v) if isinstance(v, tuple) else v) for k, v in self.__dict__.items()}


def _agreement(ratios: np.ndarray) -> tuple[float, float]:
    if ratios.size == 0:
        return 0.0, 0.0
    med = float(np.median(ratios))
    if ratios.size < MIN_PAIRS_FOR_AGREEMENT or med <= 0:
        return med, 0.0
    q1, q3 = np.quantile(ratios, [0.25, 0.75], method="weibull")
    return med, med / (med + float(q3 - q1))


def comparison_from_samples(base: Sequence[float], cand: Sequence[float]) -> PairedComparison:
    """Summarise aligned baseline/candidate observations (ms)."""
    b = np.asarray(base, dtype=np.float64).reshape(-1)
    c = np.asarray(cand, dtype=np.float64).reshape(-1)
    if b.size == 0 or b.size != c.size:
        raise ValueError(f"paired samples need two nonempty arrays of one length (got {b.size} and {c.size})")
    d = b - c
    n = int(d.size)
    if n == 1:
        spread = float("inf")
    elif np.isfinite(d).all():
        spread = float(np.std(d, ddof=1))
    else:
        spread = float("nan")  # a non-finite sample: the comparison can never resolve
    keep = b > 0
    ratios = c[keep] / b[keep]
    med_ratio, agree = _agreement(ratios)
    return PairedComparison(
        baseline_ms=tuple(b.tolist()), candidate_ms=tuple(c.tolist()), deltas_ms=tuple(d.tolist()),
        median_baseline_ms=float(np.median(b)), median_delta_ms=float(np.median(d)), spread_ms=spread,
        sigma_ms=MEDIAN_SE_FACTOR * spread / np.sqrt(n), n=n, ratios=tuple(ratios.tolist()),
        median_ratio=med_ratio, stability=agree)


def workload_win(comparisons: Mapping[str, PairedComparison], target_workload: str | None = None) -> bool:
    """True when some measured workload resolves as a win and none resolves as
    a loss. With a nominated target, that target itself must win. A
    malformed or non-finite comparison anywhere vetoes the result."""
    if not comparisons or not all(c.well_formed() for c in comparisons.values()):
        return False
    verdicts = {name: decision(c.median_delta_ms, c.sigma_ms, 0.0) for name, c in comparisons.items()}
    if min(verdicts.values()) < 0:
        return False
    if target_workload is not None:
        return verdicts.get(target_workload, 0) > 0
    return max(verdicts.values()) > 0


def paired_means(values: Sequence[float]) -> list[float]:
    """Collapse a forward/reverse block sequence (A then A again in reverse
    order) into one observation per block: the mean of its two samples."""
    v = np.asarray(values, dtype=np.float64).reshape(-1)
    if v.size < 2 or v.size % 2:
        raise ValueError(f"block samples come in pairs; got {v.size}")
    return v.reshape(-1, 2).mean(axis=1).tolist()
