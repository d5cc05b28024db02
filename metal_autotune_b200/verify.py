"""Candidate verification fanned out one workload per GPU, with host-side
failure detection (the reference's sandbox: one worker process per
evaluation, autotuner/sandbox/protocol.py:179-238, and its GPU-window
watchdog, autotuner/sandbox/watchdog.py:7-31).

A verification job is one bundle checked in a fresh worker process
(bundles/artifact.validate: original vs bundle-applied target on the
bundle's workloads), or one candidate kernel climbing the verification
ladder (ladder.run_ladder on the LadderJob a named builder returns in the
worker), as the reference's sandbox runs each evaluation in its own child. `fan_out` runs the jobs on the given GPUs, at most one
worker per GPU at a time (CUDA_VISIBLE_DEVICES pins each worker), and
returns one Verdict per job. No collective: the jobs are independent.

Supervision (`supervise`): the worker gets a dedicated pipe (its fd in
MT_WATCHDOG_FD) and writes b"B" when GPU work begins and b"E" when it ends
(`gpu_window`, nesting-safe: an inner window can neither open a new deadline
nor extend the outer one). The supervisor enforces two limits:
  - a wall-clock budget for the whole worker;
  - a GPU-window deadline from the first b"B", cleared only by the matching
    b"E" (cooling, logging and large stdout outside a window never count).
A worker past either limit is killed and reported as a failed Verdict with
`abort_job` set when the stall or a crash happened inside a GPU window:
the orchestrator must stop issuing GPU work (`require_responsive`). Faults
are detected on the host only; nothing here makes a GPU fault or hang.
"""
from __future__ import annotations

import json
import os
import select
import subprocess
import sys
import tempfile
import threading
import time
from contextlib import contextmanager
from dataclasses import dataclass, field
from pathlib import Path

GPU_WINDOW_S = 60.0
WATCHDOG_ENV = "MT_WATCHDOG_FD"


# ------------------------------------------------------------------ worker side
class _Window:
    depth = 0


@contextmanager
def gpu_window():
    """Mark GPU work for the supervisor's deadline; nested windows share the
    outermost one's deadline."""
    fd = os.environ.get(WATCHDOG_ENV)
    if fd is None:
        yield
        return
    if _Window.depth == 0:
        os.write(int(fd), b"B")
    _Window.depth += 1
    try:
        yield
    finally:
        _Window.depth -= 1
        if _Window.depth == 0:
            os.write(int(fd), b"E")


# ------------------------------------------------------------------ verdicts
@dataclass
class Verdict:
    passed: bool
    job: str
    detail: dict = field(default_factory=dict)

    def to_json(self) -> str:
        return json.dumps({"passed": self.passed, "job": self.job, "detail": self.detail}, default=float)


class WorkerFailed(RuntimeError):
    """The worker crashed, could not start, or gave no verdict."""


class WorkerUnresponsive(WorkerFailed):
    """A worker stalled inside GPU work: issue no further GPU command."""


def require_responsive(v: Verdict) -> None:
    """Raise when a verdict says the job must stop (stall or crash inside a GPU window)."""
    if v.detail.get("abort_job"):
        kind = WorkerUnresponsive if v.detail.get("failure") == "gpu_timeout" else WorkerFailed
        msg = f"{v.job}: {v.detail.get('reason', '')}"
        if v.detail.get("stderr_tail"):
            msg += "\nworker stderr:\n" + v.detail["stderr_tail"]
        raise kind(msg)


def _tail(text: str, n: int = 2000) -> str:
    return text[-n:]


# ------------------------------------------------------------------ supervisor
def supervise(command: list[str], payload: str, env: dict, timeout_s: float,
              gpu_timeout_s: float = GPU_WINDOW_S, job: str = ""):
    """Run one worker; returns subprocess.CompletedProcess on a clean exit or
    a failed Verdict (timeout, stall, crash)."""
    rfd, wfd = os.pipe()
    proc = None
    try:
        with tempfile.TemporaryFile() as fin, tempfile.TemporaryFile() as fout, tempfile.TemporaryFile() as ferr:
            fin.write(payload.encode())
            fin.seek(0)
            try:
                proc = subprocess.Popen(command, stdin=fin, stdout=fout, stderr=ferr,
                                        env={**env, WATCHDOG_ENV: str(wfd)}, pass_fds=(wfd,))
            except OSError as e:
                return Verdict(False, job, {"reason": f"worker could not start: {e}", "failure": "spawn"})
            t_end = time.monotonic() + timeout_s
            gpu_end = None
            in_window = False
            why = kind = None
            while proc.poll() is None:
                now = time.monotonic()
                if gpu_end is not None and now >= gpu_end:
                    why, kind = f"GPU window exceeded {gpu_timeout_s:g} s", "gpu_timeout"
                    break
                if now >= t_end:
                    why, kind = f"worker exceeded its {timeout_s:g} s budget", "wall_timeout"
                    break
                wait = min(0.05, t_end - now, (gpu_end - now) if gpu_end is not None else 0.05)
                ready, _, _ = select.select([rfd], [], [], max(wait, 0.0))
                if ready:
                    for ev in os.read(rfd, 4096):
                        if ev == ord("B"):
                            in_window = True
                            if gpu_end is None:
                                gpu_end = time.monotonic() + gpu_timeout_s
                        elif ev == ord("E"):
                            in_window = False
                            gpu_end = None
            if why is not None:
                proc.kill()
                try:
                    proc.wait(timeout=5)
                except subprocess.TimeoutExpired:
                    why += "; the worker did not exit after SIGKILL"
            # drain window events written just before a crash
            while select.select([rfd], [], [], 0)[0]:
                data = os.read(rfd, 4096)
                if not data:
                    break
                for ev in data:
                    in_window = ev == ord("B") if ev in (ord("B"), ord("E")) else in_window
            fout.seek(0)
            ferr.seek(0)
            out = fout.read().decode(errors="replace")
            err = ferr.read().decode(errors="replace")
            if why is not None:
                return Verdict(False, job, {"reason": why, "failure": kind, "abort_job": kind == "gpu_timeout",
                                            "stderr_tail": _tail(err), "worker_exited": proc.poll() is not None})
            if proc.returncode != 0 and not out.strip():
                return Verdict(False, job, {"reason": f"worker exited with {proc.returncode}", "failure": "crash",
                                            "abort_job": in_window, "stderr_tail": _tail(err)})
            return subprocess.CompletedProcess(command, proc.returncode, out, err)
    finally:
        if proc is not None and proc.poll() is None:
            proc.kill()
            try:
                proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                pass
        os.close(rfd)
        os.close(wfd)


def _verdict_from(res, job: str) -> Verdict:
    if isinstance(res, Verdict):
        return res
    for line in reversed(res.stdout.strip().splitlines()):
        try:
            d = json.loads(line)
        except json.JSONDecodeError:
            continue
        if isinstance(d, dict) and "passed" in d:
            return Verdict(bool(d["passed"]), job, d.get("detail", {}))
    return Verdict(False, job, {"reason": "worker gave no verdict line", "failure": "no_verdict",
                                "stderr_tail": _tail(res.stderr)})


# ------------------------------------------------------------------ fan-out
def fan_out(jobs: list[dict], gpus: list[int], *, timeout_s: float = 900.0, gpu_timeout_s: float = GPU_WINDOW_S,
            command: list[str] | None = None) -> list[Verdict]:
    """Run every job in its own worker, at most one worker per GPU at a time.
    A job is {"name": ..., "bundle": path}, {"name": ..., "ladder":
    "module:function", "args": [...]} (or anything a custom `command`
    worker reads from its stdin). Verdicts come back in job order. After a
    verdict with abort_job set, no further job is started."""
    if not gpus:
        raise ValueError("fan_out needs at least one GPU index")
    cmd = command or [sys.executable, "-m", "metal_autotune_b200.verify", "worker"]
    out: list[Verdict | None] = [None] * len(jobs)
    lock = threading.Lock()
    queue = list(range(len(jobs)))
    stop = threading.Event()

    def lane(gpu: int):
        while not stop.is_set():
            with lock:
                if not queue:
                    return
                i = queue.pop(0)
            job = jobs[i]
            env = {**os.environ, "CUDA_VISIBLE_DEVICES": str(gpu)}
            v = _verdict_from(supervise(cmd, json.dumps(job), env, timeout_s, gpu_timeout_s, job.get("name", "")),
                              job.get("name", ""))
            v.detail.setdefault("gpu", gpu)
            out[i] = v
            if v.detail.get("abort_job"):
                stop.set()

    threads = [threading.Thread(target=lane, args=(g,), daemon=True) for g in gpus]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    return [v if v is not None else Verdict(False, jobs[i].get("name", ""), {"reason": "not run: the job stopped",
                                                                              "failure": "skipped"})
            for i, v in enumerate(out)]


# ------------------------------------------------------------------ worker
def _ladder_verdict(job: dict, name: str) -> Verdict:
    """A ladder job: {"ladder": "module:function", "args": [...]}; the
    function builds a ladder.LadderJob in this worker, which climbs it."""
    import importlib

    from . import ladder
    module, _, fn = job["ladder"].partition(":")
    build = getattr(importlib.import_module(module), fn)
    with gpu_window():
        res = ladder.run_ladder(build(*job.get("args", [])))
    return Verdict(res.passed, name, {"failed_gate": res.failed_gate, "gates_passed": list(res.gates_passed),
                                      "detail": res.detail, "info": res.info})


def _worker() -> int:
    job = json.loads(sys.stdin.read() or "{}")
    name = job.get("name", "")
    try:
        if "ladder" in job:
            print(_ladder_verdict(job, name).to_json(), flush=True)
            return 0
        with gpu_window():
            from .bundles import artifact
            checks = artifact.validate(Path(job["bundle"]))
        passed = bool(checks) and all(c["passed"] for c in checks)
        print(Verdict(passed, name, {"checks": checks}).to_json(), flush=True)
        return 0
    except Exception as e:  # a failed evaluation is a verdict, not a crash
        print(Verdict(False, name, {"reason": f"{type(e).__name__}: {e}", "failure": "exception"}).to_json(),
              flush=True)
        return 0


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "worker":
        sys.exit(_worker())
    import argparse
    ap = argparse.ArgumentParser(prog="python -m metal_autotune_b200.verify")
    ap.add_argument("bundles", nargs="+", type=Path)
    ap.add_argument("--gpus", default="0", help="comma-separated GPU indices")
    a = ap.parse_args()
    vs = fan_out([{"name": b.name, "bundle": str(b)} for b in a.bundles], [int(g) for g in a.gpus.split(",")])
    for v in vs:
        print(v.to_json())
    sys.exit(0 if all(v.passed for v in vs) else 1)
