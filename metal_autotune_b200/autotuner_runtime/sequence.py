"""Consecutive model calls and tokens/s (the reference's
autotuner_runtime/sequence.py:16-188), timed with CUDA events."""
from __future__ import annotations

import statistics
from typing import Callable

from .measure import Session
from .stats import comparison_from_samples


def generation_throughput(row: dict) -> dict:
    """Generated tokens per total request second, prompt processing included
    (sequence.py:16-24)."""
    if row.get("workload_kind") != "library_generation":
        return {}
    n = row["steps"]
    return {"baseline_tokens_per_second": n * 1000 / row["baseline_sequence_ms"],
            "candidate_tokens_per_second": n * 1000 / row["candidate_sequence_ms"]}


def throughput_text(row: dict) -> str:
    r = generation_throughput(row)
    if not r:
        return ""
    return (f"generated tokens/sec: baseline {r['baseline_tokens_per_second']:.2f}, "
            f"optimized {r['candidate_tokens_per_second']:.2f} "
            "(includes prompt processing; not decode-only throughput)")


def make_sequence(step: Callable, inputs: list, steps: int) -> Callable[[], list]:
    """`steps` consecutive calls on the same inputs; every call's outputs are
    returned so none can be dropped as dead work (sequence.py:34-60). On one
    CUDA stream the calls already run back to back."""
    if isinstance(steps, bool) or not isinstance(steps, int) or steps < 1:
        raise ValueError("sequence steps must be a positive integer")

    def run():
        return [step(*inputs) for _ in range(steps)]
    run.steps = steps  # type: ignore[attr-defined]
    return run


def compare_sequences(session: Session, baseline: Callable, candidate: Callable, *, pairs: int = 4,
                      warmup_steps: int = 3, label: str = "sequence") -> dict:
    """Balanced AB / BA whole-sequence comparison (sequence.py:66-149)."""
    if pairs < 4 or pairs % 2 or warmup_steps < 1:
        raise ValueError("sequences need an even number of pairs >= 4 and positive warmup steps")
    warm = warmup_steps
    for fn in (baseline, candidate):
        warm = max(warm, len(session.warm_until_stable(fn)) + 1)
    base, cand, obs = [], [], []
    for p in range(pairs):
        order = ("baseline", "candidate") if p % 2 == 0 else ("candidate", "baseline")
        for arm in order:
            fn = baseline if arm == "baseline" else candidate
            for _ in range(warm):
                session.timed(fn)
            ms = session.timed(fn) * getattr(fn, "steps", 1)
            (base if arm == "baseline" else cand).append(ms)
            obs.append({"pair": p, "arm": arm, "elapsed_ms": ms})
            session.log("sequence_done", workload=label, **obs[-1])
        session.settle()
    cmp = comparison_from_samples(base, cand)
    return {
        "protocol": "whole_sequences_balanced_ab_ba", "warmup_steps": warm, "pairs": pairs,
        "observations": obs, "timing": cmp.as_record(),
        "baseline_sequence_ms": cmp.median_baseline_ms, "candidate_sequence_ms": statistics.median(cand),
        "speedup": 1 / cmp.median_ratio if cmp.median_ratio else float("nan"),
        "latency_reduction_pct": 100 * (1 - cmp.median_ratio),
        "win_confirmed": cmp.wins_by(0.0), "regression_confirmed": cmp.loses_by(0.0),
    }


BenchSession = Session
