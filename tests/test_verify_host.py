"""Host-side failure detection of the verification fan-out
(metal_autotune_b200/verify.py), with fake workers: plain Python processes
that write the GPU-window events to the watchdog pipe, sleep, crash or exit.
No GPU is touched: the stalls and crashes are made on the host."""
from __future__ import annotations

import json
import os
import subprocess
import sys
import time
from pathlib import Path

import pytest

from metal_autotune_b200 import verify

PRE = "import os, sys, time, json; fd = int(os.environ['MT_WATCHDOG_FD']); job = json.loads(sys.stdin.read()); "


def run(code, *, timeout=5.0, gpu_timeout=0.2):
    return verify.supervise([sys.executable, "-c", PRE + code], "{}", dict(os.environ), timeout, gpu_timeout, "t")


def test_stall_inside_gpu_window_is_killed_fast_and_aborts():
    t0 = time.monotonic()
    v = run("os.write(fd, b'B'); time.sleep(30)")
    assert time.monotonic() - t0 < 3
    assert isinstance(v, verify.Verdict) and not v.passed
    assert v.detail["failure"] == "gpu_timeout" and v.detail["abort_job"]
    with pytest.raises(verify.WorkerUnresponsive):
        verify.require_responsive(v)


def test_nested_windows_cannot_extend_the_deadline():
    v = run("os.write(fd, b'B'); time.sleep(0.15); os.write(fd, b'B'); time.sleep(0.15); time.sleep(5)")
    assert isinstance(v, verify.Verdict) and v.detail["abort_job"]


def test_time_between_windows_does_not_count():
    r = run("os.write(fd, b'BE'); time.sleep(0.5); os.write(fd, b'BE'); print('done')")
    assert isinstance(r, subprocess.CompletedProcess) and r.stdout.strip() == "done"


def test_large_stdout_cannot_block_the_deadline():
    v = run("os.write(fd, b'B'); print('x' * 2_000_000, flush=True); time.sleep(30)")
    assert isinstance(v, verify.Verdict) and v.detail["abort_job"]


def test_wall_budget_limits_work_outside_windows():
    v = run("time.sleep(30)", timeout=0.3)
    assert isinstance(v, verify.Verdict) and v.detail["failure"] == "wall_timeout" and not v.detail["abort_job"]


def test_crash_inside_a_window_aborts_the_job():
    v = run("os.write(fd, b'B'); time.sleep(0.05); os._exit(9)")
    assert isinstance(v, verify.Verdict) and v.detail["failure"] == "crash" and v.detail["abort_job"]
    with pytest.raises(verify.WorkerFailed):
        verify.require_responsive(v)


def test_crash_outside_a_window_is_a_failed_job_only():
    v = run("os.write(fd, b'BE'); os._exit(3)")
    assert isinstance(v, verify.Verdict) and not v.detail["abort_job"]
    verify.require_responsive(v)


def _fake_worker(body):
    return [sys.executable, "-c", PRE + body]


def test_fan_out_one_worker_per_gpu_and_verdicts_in_job_order():
    body = ("os.write(fd, b'B'); time.sleep(job['t']); os.write(fd, b'E'); "
            "print(json.dumps({'passed': job['ok'], 'detail': {'cvd': os.environ['CUDA_VISIBLE_DEVICES'], "
            "'start': time.time()}}))")
    jobs = [{"name": f"j{i}", "t": 0.3, "ok": i != 2} for i in range(4)]
    t0 = time.monotonic()
    vs = verify.fan_out(jobs, [0, 1], timeout_s=10, gpu_timeout_s=5, command=_fake_worker(body))
    elapsed = time.monotonic() - t0
    assert [v.job for v in vs] == ["j0", "j1", "j2", "j3"]
    assert [v.passed for v in vs] == [True, True, False, True]
    assert {v.detail["cvd"] for v in vs} == {"0", "1"}
    assert all(v.detail["cvd"] == str(v.detail["gpu"]) for v in vs)
    assert elapsed < 4 * 0.3 + 1.5  # two lanes in parallel, not four serial jobs plus slack


def test_fan_out_stops_after_an_unresponsive_worker():
    body = ("os.write(fd, b'B'); time.sleep(30 if job['stall'] else 0.01); os.write(fd, b'E'); "
            "print(json.dumps({'passed': True}))")
    jobs = [{"name": "a", "stall": True}] + [{"name": f"b{i}", "stall": False} for i in range(3)]
    vs = verify.fan_out(jobs, [0], timeout_s=10, gpu_timeout_s=0.2, command=_fake_worker(body))
    assert vs[0].detail["abort_job"]
    assert all(v.detail.get("failure") == "skipped" for v in vs[1:])


def test_worker_without_a_verdict_line_fails():
    vs = verify.fan_out([{"name": "x"}], [0], command=_fake_worker("print('no json here')"))
    assert not vs[0].passed and vs[0].detail["failure"] == "no_verdict"


def test_ladder_job_climbs_in_its_own_worker(monkeypatch):
    """A ladder job names a builder; the worker builds the LadderJob and runs
    the ladder. Static failures need no GPU, so two zoo cheats stopped at
    gate 1 check the whole round trip on the host."""
    tests_dir = str(Path(__file__).resolve().parent)
    root = str(Path(__file__).resolve().parents[1])
    monkeypatch.setenv("PYTHONPATH", os.pathsep.join([tests_dir, root, os.environ.get("PYTHONPATH", "")]))
    jobs = [{"name": n, "ladder": "ladder_cheats:zoo_job", "args": [n, "cpu"]}
            for n in ("fallback_missing", "live_output_dropping")]
    vs = verify.fan_out(jobs, [0], timeout_s=300)
    assert [v.job for v in vs] == ["fallback_missing", "live_output_dropping"]
    for v in vs:
        assert not v.passed and v.detail["failed_gate"] == "static", v.detail
        assert v.detail["gates_passed"] == []
    assert [f["check"] for f in vs[0].detail["detail"]["failures"]] == ["fallback_missing"]
    assert "live_output_dropped" in [f["check"] for f in vs[1].detail["detail"]["failures"]]
