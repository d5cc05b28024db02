"""The cheat zoo for the verification ladder: candidates that are wrong in one
particular way, each with the gate that must stop it (the reference's
tests/cheats/__init__.py:237-247 maps its Metal cheats the same way).

Most cheats are the Qwen3 RMSNorm region spec (mt_rms_norm) with one lie in
its launch record; all of them stay in bounds: a cheat writes fewer rows or
reads the right-sized buffer in the wrong order, never past an allocation.
Two cheats have no libmt counterpart and are torch stand-ins
(candidate(inputs, init_value)): a racy float-atomic row sum and a
sequential half-precision accumulator. Every builder returns
(candidate, gate, what it does).
"""
from __future__ import annotations

from dataclasses import replace

import torch

from metal_autotune_b200.bundles import qwen3_specs
from metal_autotune_b200.ladder import EvalSet, LadderJob, RegionContract

EPS = 1e-6
ROWS, DIM = 64, 2048          # primary workload: 64 tokens of a 2048-wide hidden state


def rms_norm_spec():
    return next(s for s in qwen3_specs(eps=EPS) if s.kernel_id == "rms_norm")


def _with_arg(spec, index: int, arg: dict, **changes):
    args = list(spec.cuda["args"])
    args[index] = arg
    return replace(spec, cuda={**spec.cuda, "args": args}, **changes)


def rms_norm_original(inputs):
    """The region's original ops (Qwen3 RMSNorm: fp32 statistics, one rounding)."""
    x, w = inputs
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)
    return [(xf * r * w.float()).to(x.dtype)]


def add_rms_norm_original(inputs):
    """Residual add then RMSNorm: both the sum and the normalised value are live."""
    x, res, w = inputs
    h = x + res
    return [h, rms_norm_original([h, w])[0]]


def rms_norm_sets(device, dtype=torch.bfloat16, seed=0) -> list:
    """The primary workload (two input sets at one size), a workload set at
    another size, and two correctness-only sweep sizes (one larger than the
    hard-coded cheat's 64 rows, one ragged)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    w = (1 + 0.1 * torch.randn(DIM, generator=g)).to(dtype).to(device)

    def x(rows):
        return torch.randn(rows, DIM, generator=g).to(dtype).to(device)

    return [EvalSet("primary", [[x(ROWS), w], [x(ROWS), w]]),
            EvalSet("rows16", [[x(16), w]]),
            EvalSet("rows256", [[x(256), w]], correctness_only=True),
            EvalSet("rows3", [[x(3), w]], correctness_only=True)]


def rms_norm_job(candidate, device, *, requires_fallback=False) -> LadderJob:
    sets = rms_norm_sets(device)
    contract = RegionContract.traced(rms_norm_original, sets[0].input_sets[0], requires_fallback=requires_fallback)
    return LadderJob(candidate, rms_norm_original, contract, sets, weights=(False, True))


# ----------------------------------------------------------------- the cheats
def partial_write():
    return _with_arg(rms_norm_spec(), 4, {"expr": "in0.shape[0] // 2"}), "poison", (
        "normalises only the first half of the rows; the NaN-filled output keeps NaN in the rest")


def shape_hardcoded():
    return _with_arg(rms_norm_spec(), 4, {"expr": "min(in0.shape[0], 64)"}), "sweep", (
        "bakes the primary row count into its launch: right at 64 rows and below, rows past 64 "
        "left unwritten at the 256-row sweep size")


def stride_lying():
    return replace(rms_norm_spec(), ensure_row_contiguous=False), "sweep", (
        "right math on a raw buffer: the transposed-layout inputs reach it uncopied and it reads "
        "them in storage order")


def eps_dropping():
    return _with_arg(rms_norm_spec(), 2, {"float": 0.0}), "smoke", (
        "drops the 1e-6 under the square root: indistinguishable on the recorded values, wrong by "
        "a factor of ten once inputs are scaled down by 1e-4")


def fallback_declared_but_dead():
    spec, _, _ = shape_hardcoded()
    return replace(spec, fallback_predicate="in0.shape[0] > 100000"), "sweep", (
        "the hard-coded row count plus a fallback predicate that no sweep size reaches")


def fallback_missing():
    return rms_norm_spec(), "static", (
        "a shape-specialised candidate (the contract requires a fallback) that declares none")


def live_output_dropping():
    spec = rms_norm_spec()
    args = [{"in": 0}, {"in": 2}, {"float": EPS}, {"out": 0}, {"expr": "in0.shape[0]"},
            {"expr": "in0.shape[1]"}, {"dtype": "in0"}, {"stream": True}]
    spec = replace(spec, kernel_id="cheat_live_output_dropped", input_names=("in0", "in1", "in2"),
                   cuda={"symbol": "mt_rms_norm", "args": args})
    return spec, "static", (
        "produces one output against a residual-add region whose sum is live as well")


def cached_by_shape(stored: torch.Tensor):
    def candidate(inputs, init_value):
        return [stored.clone()]
    return candidate, "smoke", (
        "replays the stored output of the primary workload's first input set: exact there, wrong "
        "on its second input set")


# the torch stand-ins, on row-sum regions of their own
def row_sum_original(inputs):
    return [inputs[0].sum(-1)]


def fp16_sloppy_accumulation():
    def candidate(inputs, init_value):
        x = inputs[0]
        acc = torch.zeros(x.shape[0], dtype=torch.float16, device=x.device)
        for k in range(x.shape[1]):
            acc = acc + x[:, k]          # rounded to half after every term
        return [acc]
    return candidate, "smoke", (
        "a sequential half-precision accumulator: over 8192 terms of mean 0.5 the sum stalls at "
        "2048, where the next term is under half a unit in the last place")


def fp16_sum_job(candidate, device) -> LadderJob:
    g = torch.Generator(device="cpu").manual_seed(1)
    x = torch.rand(16, 8192, generator=g).half().to(device)
    sets = [EvalSet("primary", [[x]])]
    return LadderJob(candidate, row_sum_original, RegionContract.traced(row_sum_original, [x]), sets,
                     exact=False)


def atomic_racy():
    def candidate(inputs, init_value):
        x = inputs[0]
        rows = torch.arange(x.shape[0], device=x.device).repeat_interleave(x.shape[1])
        out = torch.zeros(x.shape[0], dtype=x.dtype, device=x.device)   # atomics accumulate from zero
        return [out.index_add_(0, rows, x.reshape(-1))]
    return candidate, "determinism", (
        "a float-atomic row sum: within tolerance on every value gate, but the order of the adds "
        "changes from run to run, so three runs are never bitwise identical")


def atomic_sum_job(candidate, device) -> LadderJob:
    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(32, 16384, generator=g).to(device)
    sets = [EvalSet("primary", [[x]])]
    return LadderJob(candidate, row_sum_original, RegionContract.traced(row_sum_original, [x]), sets,
                     exact=False, tolerances=(1e-3, 1e-2))


# name -> (job builder on a device, the gate that must stop it); None: passes every gate
def _spec_job(builder, **kw):
    return lambda device: rms_norm_job(builder()[0], device, **kw)


def _live_output_job(device):
    g = torch.Generator().manual_seed(5)
    x, r = (torch.randn(ROWS, DIM, generator=g).bfloat16().to(device) for _ in range(2))
    w = torch.ones(DIM, dtype=torch.bfloat16, device=device)
    contract = RegionContract.traced(add_rms_norm_original, [x, r, w])
    return LadderJob(live_output_dropping()[0], add_rms_norm_original, contract, [EvalSet("primary", [[x, r, w]])])


def _cached_job(device):
    job = rms_norm_job(None, device)
    job.candidate = cached_by_shape(rms_norm_original(job.eval_sets[0].input_sets[0])[0])[0]
    job.exact = True
    return job


ZOO = {
    "correct": (lambda device: rms_norm_job(rms_norm_spec(), device), None),
    "partial_write": (_spec_job(partial_write), "poison"),
    "shape_hardcoded": (_spec_job(shape_hardcoded), "sweep"),
    "stride_lying": (_spec_job(stride_lying), "sweep"),
    "eps_dropping": (_spec_job(eps_dropping), "smoke"),
    "fallback_declared_but_dead": (_spec_job(fallback_declared_but_dead), "sweep"),
    "fallback_missing": (_spec_job(fallback_missing, requires_fallback=True), "static"),
    "live_output_dropping": (_live_output_job, "static"),
    "cached_by_shape": (_cached_job, "smoke"),
    "fp16_sloppy_accumulation": (lambda device: fp16_sum_job(fp16_sloppy_accumulation()[0], device), "smoke"),
    "atomic_racy": (lambda device: atomic_sum_job(atomic_racy()[0], device), "determinism"),
}


def zoo_job(name: str, device: str = "cuda") -> LadderJob:
    """The ladder job of a zoo entry (the builder a verification worker calls)."""
    return ZOO[name][0](device)
