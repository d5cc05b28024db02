"""Timing harness on CUDA events (the reference's autotuner/measure/ —
session.py:22-249, clocks.py:26-287 — re-hosted from host wall clocks on
Apple GPUs to device events on B200).

 - time_once / time_steps: synchronise, record a start event, run (once or
   `steps` times back to back), record an end event on the same stream,
   synchronise; device milliseconds. bench.py times its steps with these.
 - Session.warm_until_stable: throw the first call away, then sample until
   the reading stops improving by more than max(1% of best, 100 us) for 10
   samples, at most 60 (session.py:52-70, sequence.py:152-188).
 - Session.settle: the reference's duty-cycle cooling is an Apple thermal
   workaround; on B200 it only runs when duty_idle_factor > 0.
 - compare: balanced ABBA / BAAB blocks, one paired observation per block
   (clocks.py:234-287, stats.paired_means).
 - chained_loop: n calls back to back inside one timed region; stream order
   already serialises them, so no dependency link is needed.
 - loop_iterations: calls per sample so one sample lasts ~20 ms (clocks.py:129-163).
 - L2Flush: writes a buffer larger than the 126 MB L2 between samples (the
   128 MB rotation of clocks.py:48-75, sized for B200).
"""
from __future__ import annotations

import time
from typing import Callable

import torch

from .stats import PairedComparison, comparison_from_samples, paired_means


def _sync() -> None:
    torch.cuda.synchronize()


def time_steps(fn: Callable[[], object], steps: int = 1, stream: torch.cuda.Stream | None = None) -> float:
    """Device milliseconds of `steps` back-to-back calls of fn, between two
    CUDA events recorded on `stream` (default: the current stream, which is
    where fn launches its work), with the device synchronised on both sides."""
    if steps < 1:
        raise ValueError("steps must be >= 1")
    s = stream if stream is not None else torch.cuda.current_stream()
    _sync()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(s)
    for _ in range(steps):
        fn()
    end.record(s)
    _sync()
    return start.elapsed_time(end)


def time_once(fn: Callable[[], object]) -> float:
    """Device milliseconds of one call, events on the current stream."""
    return time_steps(fn, 1)


class L2Flush:
    """A buffer larger than L2; flush() overwrites it on the current stream."""

    def __init__(self, nbytes: int = 256 << 20, device=None):
        self.buf = torch.empty(nbytes // 4, dtype=torch.int32, device=device or "cuda")

    def flush(self) -> None:
        self.buf.fill_(0x5A5A5A5A)


def loop_iterations(single_ms: float, target_ms: float = 20.0, cap: int = 10_000) -> int:
    if single_ms <= 0:
        return cap
    return max(1, min(cap, int(round(target_ms / single_ms))))


def chained_loop(fn: Callable[[], object], n: int) -> Callable[[], None]:
    def run():
        for _ in range(n):
            fn()
    run.steps = n  # type: ignore[attr-defined]
    return run


class Session:
    WARM_STABLE_RTOL = 0.01
    WARM_STABLE_ABS_MS = 0.1
    WARM_CAP = 60
    WARM_PATIENCE = 10

    def __init__(self, duty_idle_factor: float = 0.0, flush: L2Flush | None = None,
                 sleep: Callable[[float], None] = time.sleep, log: Callable[..., None] | None = None,
                 clock: Callable[[Callable[[], object]], float] = time_once):
        """clock(fn) -> milliseconds of one call of fn; CUDA events by default
        (a test passes a scripted clock to drive the protocol without a GPU)."""
        self.duty_idle_factor = duty_idle_factor
        self.flush = flush
        self._sleep = sleep
        self._debt_ms = 0.0
        self._log = log
        self._clock = clock

    def timed(self, fn: Callable[[], object]) -> float:
        """Milliseconds per call of fn (a chained loop reports per step)."""
        if self.flush is not None:
            self.flush.flush()
        ms = self._clock(fn)
        self._debt_ms += ms
        return ms / getattr(fn, "steps", 1)

    def settle(self) -> None:
        if self.duty_idle_factor <= 0 or self._debt_ms <= 0:
            self._debt_ms = 0.0
            return
        idle = self.duty_idle_factor * self._debt_ms / 1000.0
        self._debt_ms = 0.0
        self._sleep(idle)

    def warm_until_stable(self, fn: Callable[[], object]) -> list[float]:
        self.timed(fn)
        times: list[float] = []
        best = None
        stale = 0
        for _ in range(self.WARM_CAP):
            t = self.timed(fn)
            times.append(t)
            improved = best is None or best - t > max(self.WARM_STABLE_RTOL * best, self.WARM_STABLE_ABS_MS)
            stale = 0 if improved else stale + 1
            best = t if best is None else min(best, t)
            if stale >= self.WARM_PATIENCE:
                break
        return times

    def log(self, kind: str, **row) -> None:
        if self._log is not None:
            self._log(kind, **row)


def compare(session: Session, baseline: Callable[[], object], candidate: Callable[[], object],
            pairs: int = 4) -> PairedComparison:
    """ABBA / BAAB blocks: each block yields a baseline and a candidate
    observation centred on the same moment."""
    if pairs < 2 or pairs % 2:
        raise ValueError("pairs must be an even number >= 2")
    session.warm_until_stable(baseline)
    session.warm_until_stable(candidate)
    base, cand = [], []
    for p in range(pairs):
        order = ("b", "c", "c", "b") if p % 2 == 0 else ("c", "b", "b", "c")
        for arm in order:
            ms = session.timed(baseline if arm == "b" else candidate)
            (base if arm == "b" else cand).append(ms)
        session.settle()
    return comparison_from_samples(paired_means(base), paired_means(cand))
