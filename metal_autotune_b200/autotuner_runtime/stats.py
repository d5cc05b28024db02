"""Paired timing comparison and its summary statistics (the reference's
autotuner_runtime/stats.py:1-102). Sign convention: a positive delta means
the candidate is faster.

A win must clear max(margin, 3 standard errors of the median delta); the
standard error of a median of normal noise is about 1.2533 sigma/sqrt(n).
The drift-immune summary is the median of per-pair ratios, with a 0..1
agreement score median / (median + IQR).
"""
from __future__ import annotations

import statistics
from dataclasses import dataclass
from math import isfinite
from typing import Mapping, Sequence

MEDIAN_SE_FACTOR = 1.2533


@dataclass(frozen=True)
class PairedComparison:
    baseline_ms: tuple[float, ...]
    candidate_ms: tuple[float, ...]
    deltas_ms: tuple[float, ...]      # per pair baseline - candidate
    median_baseline_ms: float
    median_delta_ms: float
    spread_ms: float                  # stdev of the deltas
    sigma_ms: float                   # standard error of the median delta
    n: int
    ratios: tuple[float, ...] = ()    # per pair candidate / baseline
    median_ratio: float = 0.0
    stability: float = 0.0

    def wins_by(self, margin_ms: float) -> bool:
        return self.median_delta_ms > max(margin_ms, 3.0 * self.sigma_ms)

    def loses_by(self, margin_ms: float) -> bool:
        return -self.median_delta_ms > max(margin_ms, 3.0 * self.sigma_ms)


def _finite_and_sized(c: PairedComparison) -> bool:
    if not c.n or not (len(c.baseline_ms) == len(c.candidate_ms) == len(c.deltas_ms) == c.n):
        return False
    vals = (*c.baseline_ms, *c.candidate_ms, *c.deltas_ms, *c.ratios, c.median_baseline_ms, c.median_delta_ms,
            c.spread_ms, c.sigma_ms, c.median_ratio, c.stability)
    return all(isfinite(v) for v in vals)


def workload_win(comparisons: Mapping[str, PairedComparison], target_workload: str | None = None) -> bool:
    """A resolved win and no resolved regression among the measured workloads
    (stats.py:40-63); a nominated target must win itself; invalid numbers never win."""
    if not comparisons:
        return False
    for c in comparisons.values():
        if not _finite_and_sized(c) or c.loses_by(0.0):
            return False
    if target_workload is not None:
        t = comparisons.get(target_workload)
        return t is not None and t.wins_by(0.0)
    return any(c.wins_by(0.0) for c in comparisons.values())


def ratio_stats(base: Sequence[float], cand: Sequence[float]) -> tuple[tuple[float, ...], float, float]:
    ratios = tuple(c / b for b, c in zip(base, cand) if b > 0)
    if not ratios:
        return (), 0.0, 0.0
    med = statistics.median(ratios)
    if len(ratios) < 4 or med <= 0:
        return ratios, med, 0.0
    q1, _, q3 = statistics.quantiles(ratios, n=4)
    return ratios, med, med / (med + (q3 - q1))


def paired_means(values: Sequence[float]) -> list[float]:
    """One observation per forward/reverse block (stats.py:84-88)."""
    if len(values) < 2 or len(values) % 2:
        raise ValueError("samples must contain complete forward/reverse blocks")
    return [(values[i] + values[i + 1]) / 2 for i in range(0, len(values), 2)]


def comparison_from_samples(base: Sequence[float], cand: Sequence[float]) -> PairedComparison:
    if not base or len(base) != len(cand):
        raise ValueError("comparison needs equally sized, nonempty sample sets")
    deltas = [a - b for a, b in zip(base, cand)]
    if not all(isfinite(d) for d in deltas):
        spread = float("nan")  # statistics.stdev cannot take non-finite samples; NaN never wins
    else:
        spread = statistics.stdev(deltas) if len(deltas) > 1 else float("inf")
    ratios, med_ratio, stability = ratio_stats(base, cand)
    return PairedComparison(
        baseline_ms=tuple(base), candidate_ms=tuple(cand), deltas_ms=tuple(deltas),
        median_baseline_ms=statistics.median(base), median_delta_ms=statistics.median(deltas),
        spread_ms=spread, sigma_ms=MEDIAN_SE_FACTOR * spread / len(deltas) ** 0.5, n=len(deltas),
        ratios=ratios, median_ratio=med_ratio, stability=stability)
