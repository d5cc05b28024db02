"""The verification ladder for one candidate region kernel (the reference's
autotuner/ladder/: gates.py:82 run_ladder, child.py:146-434 the gates,
static_checks.py:132-281 gate 1, numeric.py:38-78 the value regimes; the
cheat kernels each gate exists to stop are listed in its
tests/cheats/__init__.py:237-247).

A job holds the candidate, the region's original ops, the region contract
(names, ranks, dtypes, live outputs; no tolerances) and eval sets of
recorded inputs. Each eval set holds k input sets at one size; the first
eval set is the primary workload. Gates run in order, the first failure
stops:

  static       the spec against the contract, no GPU work: names, output
               arity / rank / dtype / shape at the traced size, the launch
               grammar, the fallback policy, the libmt entry point and its
               argument bindings
  compile      the first (poisoned) launch binds and runs
  poison       outputs filled with NaN before the launch: any non-finite
               value where the original's output is finite fails (an
               element the kernel never writes stays NaN)
  watchdog     candidate against original, timed with CUDA events: more
               than WATCHDOG_FACTOR times slower fails
  smoke        the primary set: every input set against the original, then
               the four value regimes (scaled down, outliers, zeros, planted
               inf / NaN lanes), references computed on the spot
  workloads    the same on every other eval set not marked correctness-only
  sweep        every correctness-only eval set (the fallback may take a
               size; a wrong size that it does not take fails, flagged
               fallback_declared_but_dead when a predicate was declared),
               then the primary inputs in a transposed layout (logically the
               same values, column-major storage)
  determinism  three re-poisoned runs bitwise identical, then the numeric
               rule on the primary set
  clock        (scoring phase, LadderJob.clock) original and candidate timed
               as interleaved loops; never fails, records whether the
               candidate ships (a resolved win over the original)

The numeric rule is exact (bit for bit) for a spec that keeps the original's
evaluation order and within tolerance for one that reassociates
(KernelSpec.reassociates; a job may force either). The original must repeat
bit for bit: a region whose own ops do not fails at determinism before any
gate runs, because widening tolerance around it would hide races.

A candidate is a KernelSpec, called through the region contract
(kernels.call, whose init_value does the poisoning), or a callable
candidate(inputs, init_value) -> outputs standing in for a kernel written
in torch ops (the racy-atomic and sloppy-accumulation cheats of the tests).
A stand-in has no spec to check statically and no kernel of its own to
time: static then checks only its outputs' count, shapes and dtypes at the
compile launch, and the watchdog is recorded as skipped. Nothing here can
fault a GPU: a wrong candidate only ever gives wrong values.
"""
from __future__ import annotations

import re
import statistics
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch

from . import lib as _mt
from .autotuner_runtime import kernels as _kernels
from .autotuner_runtime import numeric
from .autotuner_runtime.exact import bitwise_equal
from .autotuner_runtime.grammar import Expr, GrammarError

GATES = ("static", "compile", "poison", "watchdog", "smoke", "workloads", "sweep", "determinism")
DETERMINISM_RUNS = 3
WATCHDOG_FACTOR = 20.0
WATCHDOG_ITERS = 4
# the scoring phase's ninth gate (child.py:436-492): always passed, it records
# whether the candidate resolves as faster than the original
CLOCK_GATE = "clock"
CLOCK_PAIRS = 4          # ABBA / BAAB blocks
CLOCK_TARGET_MS = 20.0   # each timed arm is a loop of about this long
CLOCK_MARGIN = 0.01      # a win must beat 1% of the original's time (and 3 standard errors)

SCALE_DOWN = 1e-4
OUTLIER_VALUE = 1e4    # fits fp16 (max 65504)
OUTLIER_COUNT = 3
REGIMES = ("scaled_down", "outliers", "zeros", "nonfinite")
# The outlier regime steps down while the original's own output overflows
# where it was finite on the real data: past that, no kernel could match it.
REGIME_MAGNITUDES = {"outliers": (1e4, 1e3, 1e2)}

_C_IDENTIFIER = re.compile(r"^[A-Za-z_][A-Za-z0-9_]*$")
_TMP = re.compile(r"^tmp\d+$")
_IN_REF = re.compile(r"^in(\d+)$")


@dataclass(frozen=True)
class RegionContract:
    """The region's boundary as the static gate sees it (static_checks.py:46-62)."""
    input_names: tuple[str, ...]
    input_ranks: tuple[int, ...]
    input_dtypes: tuple[str, ...]
    output_names: tuple[str, ...]
    output_ranks: tuple[int, ...]
    output_dtypes: tuple[str, ...]
    live_outputs: tuple[str, ...]
    requires_fallback: bool = False            # the candidate is shape-specialised
    input_shapes: tuple[tuple[int, ...], ...] = ()
    output_shapes: tuple[tuple[int, ...], ...] = ()
    input_signature: list | None = None
    input_signatures: list | None = None

    @staticmethod
    def traced(original: Callable[[list], list], inputs: Sequence[torch.Tensor], *,
               live_outputs: Sequence[str] | None = None, requires_fallback: bool = False) -> "RegionContract":
        """The contract of `original` at these inputs: in0.. / out0.. names,
        the shapes and dtypes one run gives; every output live unless named."""
        outs = list(original(list(inputs)))
        names = tuple(f"out{i}" for i in range(len(outs)))
        return RegionContract(
            input_names=tuple(f"in{i}" for i in range(len(inputs))),
            input_ranks=tuple(a.dim() for a in inputs),
            input_dtypes=tuple(_kernels.dtype_name(a.dtype) for a in inputs),
            output_names=names,
            output_ranks=tuple(o.dim() for o in outs),
            output_dtypes=tuple(_kernels.dtype_name(o.dtype) for o in outs),
            live_outputs=tuple(live_outputs) if live_outputs is not None else names,
            requires_fallback=requires_fallback,
            input_shapes=tuple(tuple(a.shape) for a in inputs),
            output_shapes=tuple(tuple(o.shape) for o in outs))


@dataclass(frozen=True)
class Failure:
    check: str
    detail: str


@dataclass
class EvalSet:
    """k input sets at one size; correctness_only sets belong to the sweep."""
    label: str
    input_sets: list                        # [[tensor, ...], ...]
    correctness_only: bool = False


@dataclass
class LadderJob:
    candidate: object                       # KernelSpec or callable(inputs, init_value) -> outputs
    original: Callable[[list], list]        # the region's original ops
    contract: RegionContract
    eval_sets: list                         # [EvalSet]; [0] is the primary workload
    weights: Sequence[bool] = ()            # per input: a model weight, never perturbed
    tolerances: tuple | None = None         # (rtol, atol); None: per-output dtype defaults
    exact: bool | None = None               # None: exact unless the spec reassociates
    seed: int = 0
    clock: bool = False                     # scoring phase: run the clock gate after determinism


@dataclass
class LadderResult:
    passed: bool
    failed_gate: str | None
    detail: dict
    gates_passed: list = field(default_factory=list)
    info: dict = field(default_factory=dict)


# ----------------------------------------------------------------- value regimes
def value_regimes(inputs: Sequence[torch.Tensor], seed: int, weights: Sequence[bool] = (),
                  outlier: float = OUTLIER_VALUE) -> dict:
    """Each input under the four adversarial regimes, at its recorded shape
    (the regimes of the reference's ladder, numeric.py:38-78):

      scaled_down  every value times SCALE_DOWN
      outliers     OUTLIER_COUNT distinct elements replaced by `outlier`
      zeros        all zeros
      nonfinite    one leading-axis lane of +inf and a different one of NaN
                   (a single lane, or a scalar, becomes NaN)

    Model weights and non-float inputs (indices, masks, packed words) are
    returned as they are in every regime. Positions come from a torch
    generator seeded with (seed, input index), so a seed fixes them."""
    out = {name: [] for name in REGIMES}
    for k, a in enumerate(inputs):
        if not a.is_floating_point() or a.numel() == 0 or (k < len(weights) and weights[k]):
            for name in REGIMES:
                out[name].append(a)
            continue
        gen = torch.Generator().manual_seed(seed * 7919 + k)
        out["scaled_down"].append((a.float() * SCALE_DOWN).to(a.dtype))
        spiked = a.clone(memory_format=torch.contiguous_format)
        flat = spiked.view(-1)
        picks = torch.randperm(flat.numel(), generator=gen)[:OUTLIER_COUNT].to(flat.device)
        flat[picks] = outlier
        out["outliers"].append(spiked)
        out["zeros"].append(torch.zeros_like(a))
        lanes = a.clone()
        if lanes.dim() == 0:
            lanes.fill_(float("nan"))
        else:
            order = torch.randperm(lanes.shape[0], generator=gen).tolist()
            lanes[order[0]] = float("inf")
            lanes[order[-1]] = float("nan")   # the same lane when there is only one
        out["nonfinite"].append(lanes)
    return out


def transposed_layout(inputs: Sequence[torch.Tensor]) -> tuple[list, bool]:
    """Every input of rank >= 2 with the same values in column-major storage
    (a non-contiguous view of a transposed copy; the buffer is the same size,
    so a kernel that ignores strides reads the wrong order, never out of
    bounds). Second value: whether any input changed."""
    out, changed = [], False
    for a in inputs:
        if a.dim() >= 2:
            out.append(a.mT.contiguous().mT)
            changed = True
        else:
            out.append(a)
    return out, changed


# ----------------------------------------------------------------- gate 1
def _probe(slot: str, text: str, shapes, fails: list) -> None:
    """Parse, then evaluate at the contract's shapes, so a bad input index or
    axis fails here and not at the launch (static_checks.py:284-298)."""
    try:
        expr = Expr(text)
    except GrammarError as e:
        fails.append(Failure("launch_grammar", f"{slot}: {e}"))
        return
    try:
        expr.evaluate(shapes)
    except GrammarError as e:
        fails.append(Failure("launch_grammar", f"{slot}: {e}"))
    except ArithmeticError:
        pass  # value-dependent (a zero divisor at these sizes), not static


def _resolved_dtype(name: str, contract: RegionContract) -> str:
    m = _IN_REF.match(name)
    if m and int(m.group(1)) < len(contract.input_dtypes):
        return contract.input_dtypes[int(m.group(1))]
    return name


def _entry_point_failures(spec, n_inputs: int, n_outputs: int, shapes, where: str = "") -> list:
    """The CUDA counterpart of the reference's buffer and compile checks:
    the record names a libmt entry point, binds one argument per parameter,
    and refers only to inputs and outputs the kernel has."""
    fails: list[Failure] = []
    cuda = spec.cuda
    if cuda is None:
        return [Failure("entry_point", f"{where}no cuda record names an entry point to call")]
    sym = cuda.get("symbol")
    if sym not in _mt.SIGNATURES:
        return [Failure("entry_point", f"{where}libmt exports no {sym!r}")]
    params = _mt.SIGNATURES[sym][1]
    args = cuda.get("args", [])
    bound = sum(2 if "workspace" in a else 1 for a in args)  # a workspace is a pointer and its size
    if bound != len(params):
        fails.append(Failure("entry_point", f"{where}{sym} takes {len(params)} arguments, "
                                            f"the record binds {bound}"))
    for j, a in enumerate(args):
        if "in" in a and not 0 <= int(a["in"]) < n_inputs:
            fails.append(Failure("entry_point", f"{where}argument {j} binds input {a['in']}; "
                                                f"the kernel has {n_inputs}"))
        elif "out" in a and not 0 <= int(a["out"]) < n_outputs:
            fails.append(Failure("entry_point", f"{where}argument {j} binds output {a['out']}; "
                                                f"the kernel has {n_outputs}"))
        elif "expr" in a:
            _probe(f"{where}args[{j}]", a["expr"], shapes, fails)
    return fails


def _names(spec, contract: RegionContract, shapes):
    if not _C_IDENTIFIER.match(spec.name):
        yield Failure("kernel_name", f"name {spec.name!r} cannot be a C symbol")
    if tuple(spec.input_names) != tuple(contract.input_names):
        yield Failure("input_names", f"inputs {tuple(spec.input_names)}; the region's are "
                                     f"{tuple(contract.input_names)}")
    k = len(contract.output_names)
    extras = spec.output_names[k:]
    if tuple(spec.output_names[:k]) != tuple(contract.output_names) or any(not _TMP.match(e) for e in extras):
        yield Failure("output_names", f"outputs {tuple(spec.output_names)}: the region's "
                                      f"{tuple(contract.output_names)} first, then only tmp<N> scratch")
    for name in contract.live_outputs:
        if name not in spec.output_names:
            yield Failure("live_output_dropped", f"{name!r} is read after the region but the spec never "
                                                 "writes it")


def _outputs(spec, contract: RegionContract, shapes):
    n = len(spec.output_names)
    if (len(spec.output_shapes), len(spec.output_dtypes)) != (n, n):
        yield Failure("output_arity", f"{len(spec.output_shapes)} shapes and {len(spec.output_dtypes)} dtypes "
                                      f"for {n} outputs")
    for name, dt, want in zip(spec.output_names, spec.output_dtypes, contract.output_dtypes):
        if _resolved_dtype(dt, contract) != want:
            yield Failure("output_dtype", f"{name!r} would be {dt}; the region produces {want}")
    for name, exprs, rank in zip(spec.output_names, spec.output_shapes, contract.output_ranks):
        if len(exprs) != rank:
            yield Failure("output_rank", f"{name!r} has {len(exprs)} extents; the region's value has rank {rank}")
    probes: list[Failure] = []
    for j, exprs in enumerate(spec.output_shapes):
        for i, text in enumerate(exprs):
            _probe(f"output_shapes[{j}][{i}]", text, shapes, probes)
    yield from probes
    for name, exprs, want in zip(spec.output_names, spec.output_shapes, contract.output_shapes):
        try:
            got = tuple(Expr(e).evaluate(shapes) for e in exprs)
        except (GrammarError, ArithmeticError):
            continue  # the probe above names it
        if got != tuple(want):
            yield Failure("output_shape", f"{name!r} evaluates to {got} at the traced inputs; the region's is "
                                          f"{tuple(want)}")


def _fallback(spec, contract: RegionContract, shapes):
    if spec.fallback_predicate is None:
        if contract.requires_fallback:
            yield Failure("fallback_missing", "the candidate serves only some shapes and names no fallback "
                                              "predicate for the rest")
        return
    probes: list[Failure] = []
    _probe("fallback_predicate", spec.fallback_predicate, shapes, probes)
    yield from probes
    if probes or not contract.input_shapes:
        return
    try:
        on_primary = bool(Expr(spec.fallback_predicate).evaluate(shapes))
    except (GrammarError, ArithmeticError):
        return
    if on_primary:
        yield Failure("fallback_on_primary", "the fallback predicate holds on the primary workload, so the "
                                             "candidate would never run where it is measured")


def _launch(spec, contract: RegionContract, shapes):
    if not spec.stages:
        yield from _entry_point_failures(spec, len(spec.input_names), len(spec.output_names), shapes)
        return
    from .autotuner_runtime.stages import StageError, build_graph
    try:
        per_stage, outs = build_graph(spec).walk_shapes(shapes, [_kernels.DTYPES[d] for d in contract.input_dtypes])
    except (StageError, ValueError, ArithmeticError, GrammarError) as e:
        yield Failure("stages", str(e))
        return
    k = len(contract.output_names)
    want = [(tuple(sh), _kernels.DTYPES[d]) for sh, d in zip(contract.output_shapes, contract.output_dtypes)]
    if contract.output_shapes and [(tuple(sh), d) for sh, d in outs][:k] != want:
        yield Failure("stage_boundary", "the last stages do not produce the region's output shapes and dtypes")
    for i, (kernel, ins, outs_i) in enumerate(per_stage):
        yield from _entry_point_failures(kernel, len(ins), len(outs_i), [sh for sh, _ in ins], where=f"stage {i}: ")


_STATIC_CHECKS = (_names, _outputs, _fallback, _launch)


def static_check(spec, contract: RegionContract) -> list[Failure]:
    """Gate 1 (the reference's static_checks.py:132-281): everything a
    KernelSpec can be checked for against the region contract without a GPU,
    as a list of named failures; empty means the gate passes. A spec pinned
    to other input shapes than the contract's fails on that alone."""
    if (spec.input_signature, spec.input_signatures) != (contract.input_signature, contract.input_signatures):
        return [Failure("input_signature", "the spec pins input shapes other than those the region was "
                                           "traced with")]
    shapes = [tuple(sh) for sh in contract.input_shapes] or [(4,) * r for r in contract.input_ranks]
    return [f for check in _STATIC_CHECKS for f in check(spec, contract, shapes)]


# ----------------------------------------------------------------- gates 2-8
class _Rejected(Exception):
    """A launch the ladder refuses: the fallback takes a workload the candidate must serve."""


class _OriginalUnstable(Exception):
    """The region's original ops do not repeat bit for bit."""


def _original_outputs(job: LadderJob, inputs, n_out: int) -> list:
    """The original's outputs on `inputs`, run twice; they must agree bit for
    bit (child.py:190-201)."""
    first = [t.clone() for t in list(job.original(list(inputs)))[:n_out]]
    again = list(job.original(list(inputs)))[:n_out]
    if len(first) != len(again) or not all(bitwise_equal(a, b) for a, b in zip(first, again)):
        raise _OriginalUnstable("two runs of the region's original ops gave different bits: it is not repeatable")
    return first


def _finite_where(got: torch.Tensor, recorded: torch.Tensor) -> bool:
    """No non-finite value where the recorded output is finite."""
    if not got.is_floating_point():
        return True
    return not bool((~torch.isfinite(got) & torch.isfinite(recorded)).any())


def run_ladder(job: LadderJob) -> LadderResult:
    """Every gate in order; the first failure stops (gates.py:82, child.py:146)."""
    try:
        return _run(job)
    except _OriginalUnstable as e:
        return LadderResult(False, "determinism", {"reason": str(e)}, [], {})


def _run(job: LadderJob) -> LadderResult:
    spec = job.candidate if isinstance(job.candidate, _kernels.KernelSpec) else None
    contract = job.contract
    out_names = tuple(contract.output_names)
    n_out = len(out_names)
    exact = job.exact if job.exact is not None else not (spec is not None and spec.reassociates)
    passed: list[str] = []
    info: dict = {"correctness_rule": "exact" if exact else "tolerance", "fallback_engaged": {}}
    if not exact:
        info["tolerances"] = {n: numeric.tolerance_for(d, job.tolerances)
                              for n, d in zip(out_names, contract.output_dtypes)}
    nan = float("nan")

    def fail(gate: str, detail: dict) -> LadderResult:
        return LadderResult(False, gate, detail, passed, info)

    def launch(inputs) -> list:
        if spec is not None:
            if _kernels.fallback_fires(spec, list(inputs)):
                raise _Rejected("fallback_on_workload: the fallback predicate sends a measured workload back "
                                "to the original ops")
            return list(_kernels.call(spec, list(inputs), init_value=nan))[:n_out]
        return list(job.candidate(list(inputs), nan))

    def mismatch(got, want) -> dict | None:
        if len(got) != len(want):
            return {"reason": f"{len(got)} outputs where the region has {len(want)}"}
        for name, g, w in zip(out_names, got, want):
            rtol, atol = numeric.tolerance_for(w.dtype, job.tolerances)
            r = numeric.check(g, w, exact=exact, rtol=rtol, atol=atol)
            if not r.passed:
                return {"output": name, "reason": r.reason, "max_excess": r.max_excess,
                        "index": list(r.index) if r.index is not None else None, "note": r.detail}
        return None

    def checked(inputs) -> dict | None:
        """One candidate launch against the original on the same inputs."""
        return mismatch(launch(inputs), _original_outputs(job, inputs, n_out))

    # gate 1, static: the spec against the contract, in the parent, no GPU work
    if spec is not None:
        fails = static_check(spec, contract)
        if fails:
            return fail("static", {"failures": [{"check": f.check, "detail": f.detail} for f in fails]})
        passed.append("static")

    primary = job.eval_sets[0]
    base = primary.input_sets[0]
    # gate 2, compile: the first poisoned launch binds the entry point and runs
    try:
        outs0 = launch(base)
        torch.cuda.synchronize()
    except _Rejected as e:
        return fail("compile", {"reason": str(e)})
    except Exception as e:  # noqa: BLE001 - a launch the candidate cannot make is this gate's failure
        return fail("compile", {"probe_error": f"{type(e).__name__}: {e}"[:2000]})
    if spec is None:
        # a stand-in has no spec; its outputs carry the contract instead
        if len(outs0) != n_out:
            return fail("static", {"failures": [{"check": "live_output_dropped",
                                                 "detail": f"{len(outs0)} outputs, the region has {n_out}"}]})
        passed.append("static")
    passed.append("compile")

    # gate 3, poison: an unwritten element stays NaN
    ref0 = _original_outputs(job, base, n_out)
    counts = {}
    for name, c, r in zip(out_names, outs0, ref0):
        if tuple(c.shape) != tuple(r.shape) or c.dtype != r.dtype:
            return fail("poison", {"output": name, "reason": "shape",
                                   "note": f"{tuple(c.shape)} {c.dtype}, original {tuple(r.shape)} {r.dtype}"})
        if c.is_floating_point():
            counts[name] = int((~torch.isfinite(c) & torch.isfinite(r)).sum().item())
    if any(counts.values()):
        return fail("poison", {"non_finite_over_finite_ref": counts})
    passed.append("poison")

    # gate 4, watchdog: the candidate's device time against the original's
    if spec is not None:
        from .autotuner_runtime.measure import time_steps
        cand = lambda: _kernels.call(spec, list(base))  # noqa: E731
        orig = lambda: job.original(list(base))  # noqa: E731
        cand(), orig()
        t_cand = time_steps(cand, WATCHDOG_ITERS) / WATCHDOG_ITERS
        t_orig = time_steps(orig, WATCHDOG_ITERS) / WATCHDOG_ITERS
        info["timing"] = {"candidate_ms": t_cand, "original_ms": t_orig}
        if t_cand > WATCHDOG_FACTOR * t_orig:
            return fail("watchdog", {"candidate_ms": t_cand, "original_ms": t_orig,
                                     "watchdog_factor": WATCHDOG_FACTOR})
        passed.append("watchdog")
    else:
        info["watchdog"] = "skipped: a torch stand-in has no kernel of its own to time"

    def check_eval_set(es: EvalSet) -> dict | None:
        """Gates 5 and 6: every input set of `es`, then the value regimes on
        its first input set (child.py:308-350)."""
        for j, inputs in enumerate(es.input_sets):
            bad = checked(inputs)
            if bad:
                return {**bad, "eval_set": es.label, "input_set": j, "kind": "input_set"}
        recorded = _original_outputs(job, es.input_sets[0], n_out)
        for regime in REGIMES:
            found = None
            for magnitude in REGIME_MAGNITUDES.get(regime, (None,)):
                knobs = {} if magnitude is None else {"outlier": magnitude}
                rin = value_regimes(es.input_sets[0], job.seed, job.weights, **knobs)[regime]
                ref = _original_outputs(job, rin, n_out)
                if magnitude is None or all(_finite_where(r, w) for r, w in zip(ref, recorded)):
                    found = (rin, ref, magnitude)
                    break
            if found is None:
                info.setdefault("regime_skipped", {})[regime] = \
                    "no outlier magnitude left the original's outputs finite where they were finite"
                continue
            rin, ref, magnitude = found
            if magnitude is not None:
                info.setdefault("regime_magnitude", {})[regime] = magnitude
            bad = mismatch(launch(rin), ref)
            if bad:
                return {**bad, "eval_set": es.label, "regime": regime, "kind": "regime"}
        return None

    try:
        # gate 5, smoke: the primary workload
        bad = check_eval_set(primary)
        if bad:
            return fail("smoke", bad)
        passed.append("smoke")

        # gate 6, workloads: every other eval set that is not correctness-only
        for es in job.eval_sets[1:]:
            if not es.correctness_only:
                bad = check_eval_set(es)
                if bad:
                    return fail("workloads", bad)
        passed.append("workloads")
    except _Rejected as e:
        return fail("smoke" if "smoke" not in passed else "workloads", {"reason": str(e)})

    # gate 7, sweep: correctness-only sets with fallback routing, then the
    # transposed layout of the primary inputs
    for es in job.eval_sets[1:]:
        if not es.correctness_only:
            continue
        for j, inputs in enumerate(es.input_sets):
            fired = spec is not None and _kernels.fallback_fires(spec, list(inputs))
            key = es.label if j == 0 else f"{es.label}#{j}"
            info["fallback_engaged"][key] = fired
            want = _original_outputs(job, inputs, n_out)
            got = want if fired else launch(inputs)
            bad = mismatch(got, want)
            if bad:
                bad.update({"eval_set": es.label, "input_set": j, "kind": "sweep",
                            "fallback_engaged": dict(info["fallback_engaged"])})
                if spec is not None and spec.fallback_predicate is not None and not fired:
                    bad["fallback_declared_but_dead"] = True
                return fail("sweep", bad)
    variant, changed = transposed_layout(base)
    if changed and not (spec is not None and _kernels.fallback_fires(spec, variant)):
        # a reassociating candidate is held to the original on this layout
        # (torch's reductions may round differently over strided storage); an
        # order-keeping one reads its inputs row-contiguous and must still give
        # the recorded bits
        want = ref0 if exact else _original_outputs(job, variant, n_out)
        bad = mismatch(launch(variant), want)
        if bad:
            return fail("sweep", {**bad, "eval_set": primary.label, "kind": "transposed_layout"})
    passed.append("sweep")

    # gate 8, determinism: three re-poisoned runs bitwise identical, then the
    # numeric rule on the primary set (child.py:419-434)
    runs = [[t.clone() for t in launch(base)] for _ in range(DETERMINISM_RUNS)]
    for r_i in range(1, DETERMINISM_RUNS):
        for name, a, b in zip(out_names, runs[0], runs[r_i]):
            if not bitwise_equal(a, b):
                return fail("determinism", {"nondeterministic_output": name, "run": r_i})
    bad = mismatch(runs[0], ref0)
    if bad:
        return fail("determinism", {**bad, "eval_set": primary.label, "kind": "numeric"})
    passed.append("determinism")

    # gate 9, clock (scoring phase only): the original and the candidate as
    # loops over the primary set's input sets in turn, interleaved ABBA / BAAB
    # in one measurement session; the candidate ships when its median gain
    # beats max(CLOCK_MARGIN of the original's time, 3 standard errors)
    if job.clock:
        from .autotuner_runtime import measure
        sets = [list(x) for x in primary.input_sets]
        turn = [0]

        def arm(fn):
            def one():
                fn(sets[turn[0] % len(sets)])
                turn[0] += 1
            return one

        cand_one = arm((lambda inputs: _kernels.call(spec, inputs)) if spec is not None
                       else (lambda inputs: job.candidate(inputs, None)))
        orig_one = arm(job.original)
        single = measure.time_steps(orig_one, 4) / 4
        iters = measure.loop_iterations(single, CLOCK_TARGET_MS)
        comp = measure.compare(measure.Session(), measure.chained_loop(orig_one, iters),
                               measure.chained_loop(cand_one, iters), pairs=CLOCK_PAIRS)
        margin = CLOCK_MARGIN * comp.median_baseline_ms
        info.setdefault("timing", {}).update({
            "library_ms": comp.median_baseline_ms,
            "region_ms": statistics.median(comp.candidate_ms),
            "win_ms": comp.median_delta_ms, "sigma_ms": comp.sigma_ms,
            "clock_iters": iters, "clock_sets": len(sets), "clock_deltas": comp.n})
        info.update({"ship": comp.wins_by(margin), "margin_ms": max(margin, 3.0 * comp.sigma_ms)})
        passed.append(CLOCK_GATE)
    return LadderResult(True, None, {}, passed, info)
