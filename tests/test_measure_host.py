"""The timing harness (autotuner_runtime/measure.py, sequence.py) driven by a
scripted clock on the CPU: warm-until-stable, ABBA/BAAB pairing, duty-cycle
settling, L2 flushing between samples, loop sizing and the whole-sequence
comparison. The clock is the only GPU dependency (CUDA events), so a fake
clock exercises the whole protocol."""
from __future__ import annotations

import itertools

import pytest

from metal_autotune_b200.autotuner_runtime import measure, sequence


class ScriptedClock:
    """clock(fn) -> the next scripted time of that arm; records the call order."""

    def __init__(self, scripts):
        self.scripts = {k: iter(v) for k, v in scripts.items()}
        self.order = []

    def __call__(self, fn):
        name = fn.__name__
        self.order.append(name)
        return next(self.scripts[name])


def base():
    pass


def cand():
    pass


def test_warm_until_stable_stops_after_patience():
    # improving by 1 ms each call, then flat: stops 10 flat samples after the last improvement
    times = [50.0, 20, 19, 18, 17] + [17.0] * 100
    clock = ScriptedClock({"base": times})
    s = measure.Session(clock=clock)
    got = s.warm_until_stable(base)
    assert got[:4] == [20, 19, 18, 17]
    assert len(got) == 4 + measure.Session.WARM_PATIENCE
    assert len(clock.order) == len(got) + 1  # the first call is thrown away


def test_warm_until_stable_caps_samples():
    clock = ScriptedClock({"base": (100.0 - i for i in itertools.count())})
    got = measure.Session(clock=clock).warm_until_stable(base)
    assert len(got) == measure.Session.WARM_CAP


def test_compare_pairs_abba_blocks_and_resolves_a_win():
    clock = ScriptedClock({"base": itertools.cycle([10.0, 10.2, 9.9, 10.1]),
                           "cand": itertools.cycle([8.0, 8.1, 7.9, 8.05])})
    s = measure.Session(clock=clock)
    c = measure.compare(s, base, cand, pairs=4)
    timed = clock.order[-16:]
    assert timed == ["base", "cand", "cand", "base", "cand", "base", "base", "cand"] * 2
    assert c.n == 4 and c.wins_by(1.0) and not c.loses_by(0.0)
    assert 0.75 < c.median_ratio < 0.85


def test_compare_unresolved_when_noise_covers_the_delta():
    clock = ScriptedClock({"base": itertools.cycle([10.0, 14.0, 6.0, 10.0]),
                           "cand": itertools.cycle([9.0, 5.0, 15.0, 9.5])})
    c = measure.compare(measure.Session(clock=clock), base, cand, pairs=4)
    assert not c.wins_by(0.0) and not c.loses_by(0.0)


def test_compare_needs_even_pairs():
    with pytest.raises(ValueError):
        measure.compare(measure.Session(clock=lambda f: 1.0), base, cand, pairs=3)


def test_settle_sleeps_in_proportion_to_busy_time():
    slept = []
    s = measure.Session(duty_idle_factor=0.5, clock=lambda f: 40.0, sleep=slept.append)
    s.timed(base)
    s.timed(base)
    s.settle()
    assert slept == [pytest.approx(0.04)]
    s.settle()  # no debt left
    assert len(slept) == 1
    s0 = measure.Session(clock=lambda f: 40.0, sleep=slept.append)
    s0.timed(base)
    s0.settle()
    assert len(slept) == 1  # factor 0: never sleeps


def test_flush_runs_before_every_sample():
    class Flush:
        n = 0

        def flush(self):
            Flush.n += 1

    s = measure.Session(flush=Flush(), clock=lambda f: 1.0)
    for _ in range(5):
        s.timed(base)
    assert Flush.n == 5


def test_chained_loop_reports_per_step_time():
    calls = []
    loop = measure.chained_loop(lambda: calls.append(1), 8)
    s = measure.Session(clock=lambda f: (f(), 16.0)[1])
    assert s.timed(loop) == 2.0 and len(calls) == 8


@pytest.mark.parametrize("single,target,expect", [(0.5, 20.0, 40), (30.0, 20.0, 1), (0.0, 20.0, 10_000),
                                                  (1e-6, 20.0, 10_000)])
def test_loop_iterations(single, target, expect):
    assert measure.loop_iterations(single, target) == expect


def test_compare_sequences_balanced_and_reports_speedup():
    def seq_base():
        pass

    def seq_cand():
        pass
    seq_base.steps = seq_cand.steps = 2
    clock = ScriptedClock({"seq_base": itertools.cycle([20.0]), "seq_cand": itertools.cycle([10.0])})
    out = sequence.compare_sequences(measure.Session(clock=clock), seq_base, seq_cand, pairs=4, warmup_steps=1)
    assert out["protocol"] == "whole_sequences_balanced_ab_ba" and out["pairs"] == 4
    arms = [o["arm"] for o in out["observations"]]
    assert arms == ["baseline", "candidate", "candidate", "baseline"] * 2
    assert out["speedup"] == pytest.approx(2.0) and out["win_confirmed"]
    assert out["timing"]["n"] == 4
