"""Explicit multi-kernel dataflow of one region (the reference's
autotuner_runtime/stages.py:7-53): validated without touching tensors.

Rules: a stage reads region inputs or earlier results; its kernel uses the
local in0../out0.. ABI; outputs are new tmpN names or region outputs, never
an overwrite; the stages must produce every region output; a produced value
nobody reads is dead work that would hide from timing, so it is rejected.
"""
from __future__ import annotations

import re

from .grammar import Expr


def wiring(spec):
    """Return (buffer indices per stage, buffer index of each region output)."""
    slot = {name: i for i, name in enumerate(spec.input_names)}
    produced, read, plan = set(), set(), []
    for n, stage in enumerate(spec.stages):
        k = stage.kernel
        if k.stages:
            raise ValueError(f"stage {n}: must be a plain, non-nested kernel")
        if k.fallback_predicate is not None or k.input_signature is not None or k.input_signatures is not None:
            raise ValueError(f"stage {n}: fallback and signature policies belong to the whole region")
        missing = [x for x in stage.inputs if x not in slot]
        if missing:
            raise ValueError(f"stage {n}: inputs {missing} must name region inputs or earlier results")
        if k.input_names != tuple(f"in{j}" for j in range(len(stage.inputs))):
            raise ValueError(f"stage {n}: kernel input names must use the local inN ABI")
        if not stage.outputs or k.output_names != tuple(f"out{j}" for j in range(len(stage.outputs))):
            raise ValueError(f"stage {n}: kernel output names must use the local outN ABI")
        if len(k.output_shapes) != len(stage.outputs) or len(k.output_dtypes) != len(stage.outputs):
            raise ValueError(f"stage {n}: each output needs a shape and a dtype")
        plan.append(tuple(slot[x] for x in stage.inputs))
        read.update(stage.inputs)
        for name in stage.outputs:
            fresh = re.fullmatch(r"tmp\d+", name) or name in spec.output_names
            if name in slot or not fresh:
                raise ValueError(f"stage {n}: output {name!r} must be a new tmpN or region output")
            slot[name] = len(slot)
            produced.add(name)
    if not set(spec.output_names) <= produced:
        raise ValueError("stages must produce every region output")
    if produced - read - set(spec.output_names):
        raise ValueError("unused stage outputs would hide work from timing; remove them")
    return plan, tuple(slot[name] for name in spec.output_names)


def shapes(spec, input_shapes, input_dtypes):
    """Walk the stages in order; each stage's grammar sees its own inputs as in0..."""
    from .kernels import _resolve_dtype

    plan, outputs = wiring(spec)
    buffers = list(zip((tuple(s) for s in input_shapes), input_dtypes))
    walked = []
    for stage, idx in zip(spec.stages, plan):
        ins = [buffers[i] for i in idx]
        env = [s for s, _ in ins]
        outs = [tuple(int(Expr(e).evaluate(env)) for e in shp) for shp in stage.kernel.output_shapes]
        dts = [_resolve_dtype(d, [dt for _, dt in ins]) for d in stage.kernel.output_dtypes]
        walked.append((stage.kernel, ins, outs))
        buffers.extend(zip(outs, dts))
    return walked, [buffers[i] for i in outputs]
