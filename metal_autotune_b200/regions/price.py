"""Pricing (the reference's autotuner/regions/price.py): the region clock and
each region's share of the step, on the GPU with CUDA events.

The region clock replays one copy's recorded calls (trace.replay) on real
tensors: the module's own weights where the boundary reads a weight, seeded
random activations of the recorded shapes elsewhere (integers zero). Every
sample writes a buffer larger than the 126 MB L2 first (measure.L2Flush), so
a region is timed from HBM as it runs inside the step, then the median of
the samples is the region's time. The step is timed the same way (the
module's eager forward). p = copies x one copy's time / step time; the
roofline's s_max = one copy's time / its physical limit.

estimate() prices every region from shapes and peaks alone (no GPU): the
sum of its calls' individual limits against one fused limit, the CPU-only
ordering hint of rank.py:107-147.
"""
from __future__ import annotations

import statistics

import torch

from .build import Stretch, is_view
from .fingerprint import Region
from .roofline import Peaks, stretch_roofline
from .trace import Trace, replay

SAMPLES = 7


def _dtype(name: str) -> torch.dtype:
    return getattr(torch, name)


def bind_inputs(trace: Trace, s: Stretch, weights: dict, device, seed: int = 0) -> dict:
    """Tensors for a copy's boundary inputs: weights by path, else seeded
    random values of the recorded shape and dtype."""
    g = torch.Generator(device=device).manual_seed(seed)
    bound = {}
    for a in s.input_ids:
        if a in trace.weights:
            bound[a] = weights[trace.weights[a]]
            continue
        shape, dt = trace.specs[a]
        dtype = _dtype(dt)
        if dtype.is_floating_point:
            bound[a] = (torch.randn(shape, generator=g, device=device) * 0.5).to(dtype)
        else:
            bound[a] = torch.zeros(shape, dtype=dtype, device=device)
    return bound


def _clock(fn, flush) -> float:
    from metal_autotune_b200.autotuner_runtime import measure
    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(SAMPLES):
        flush.flush()
        times.append(measure.time_once(fn))
    return statistics.median(times)


def price(trace: Trace, regions: list[Region], module, args: tuple, pk: Peaks) -> float:
    """Fill t_rep_ms, t_orig_ms, p and roofline of every region; returns the
    step's milliseconds."""
    from metal_autotune_b200.autotuner_runtime import measure
    device = next(a.device for a in args if isinstance(a, torch.Tensor))
    weights = {}
    for prefix, sub in module.named_modules(remove_duplicate=False):
        for attr, t in list(sub._parameters.items()) + list(sub._buffers.items()):
            if t is not None:
                weights.setdefault(f"{prefix}.{attr}" if prefix else attr, t)
    flush = measure.L2Flush(device=device)
    with torch.no_grad():
        step_ms = _clock(lambda: module(*args), flush)
        for r in regions:
            s = r.members[0]
            bound = bind_inputs(trace, s, weights, device)
            t = _clock(lambda: replay(trace, s.start_seq, s.end_seq, bound), flush)
            r.t_rep_ms[trace.workload] = t
            r.t_orig_ms[trace.workload] = t * r.copies
            r.p[trace.workload] = t * r.copies / step_ms
            r.roofline = stretch_roofline(trace, s, pk, t)
    return step_ms


def estimate(trace: Trace, regions: list[Region], pk: Peaks) -> dict:
    """fingerprint -> (share of the summed per-call limits, removable part):
    unfused cost (each call's own limit) minus one fused limit, per copy."""
    per_call = []
    for node in trace.nodes:
        if is_view(node):
            per_call.append(0.0)
            continue
        s = Stretch(trace.workload, node.seq, node.seq, tuple(dict.fromkeys(node.in_arrays)),
                    tuple(dict.fromkeys(node.out_arrays)), node.module_stack)
        per_call.append(stretch_roofline(trace, s, pk).t_roofline_ms)
    total = sum(per_call) or 1.0
    out = {}
    for r in regions:
        share = removable = 0.0
        for m in r.members:
            cost = sum(per_call[m.start_seq:m.end_seq + 1])
            floor = stretch_roofline(trace, m, pk).t_roofline_ms
            share += cost / total
            removable += max(cost - floor, 0.0) / total
        out[r.fingerprint] = (share, removable)
    return out
