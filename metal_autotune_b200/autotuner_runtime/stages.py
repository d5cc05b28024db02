"""Multi-kernel regions as a typed dataflow graph over buffer slots.

A staged KernelSpec runs several libmt entry points in order. Its buffers are
numbered slots: the region inputs first, then every value a stage produces,
in production order. `build_graph` turns the spec into a `StageGraph` in one
pass over the stages and rejects, without evaluating any tensor, every plan
that breaks the contract of the reference's staged regions
(autotuner_runtime/stages.py:7-38):

  code              rule
  ----------------  -------------------------------------------------------
  nested            a stage runs one plain kernel (no stages of its own)
  stage_policy      fallback predicates and signatures belong to the region
  unbound           a stage reads only region inputs or earlier values
  local_inputs      a stage kernel names its inputs in0, in1, ... in order
  local_outputs     ... and its outputs out0, out1, ... (at least one)
  out_meta          one shape and one dtype per stage output
  rebind            a produced name is new: a tmpN or a region output
                    (inputs and earlier values are never overwritten)
  unproduced        every region output is produced by some stage
  dead              every produced value is read later or is a region
                    output (dead work would hide from the region's timing)

`walk_shapes` then evaluates each stage's output shapes with the launch
grammar, the stage's own inputs bound as in0, in1, ...
"""
from __future__ import annotations

import re
from dataclasses import dataclass

from .grammar import Expr

_TMP = re.compile(r"tmp\d+")


class StageError(ValueError):
    """A staged region that breaks the dataflow contract; `code` names the rule."""

    def __init__(self, code: str, stage: int | None, detail: str):
        where = f"stage {stage}" if stage is not None else "region"
        super().__init__(f"[{code}] {where}: {detail}")
        self.code = code
        self.stage = stage


@dataclass(frozen=True)
class StageNode:
    kernel: object                 # the stage's KernelSpec
    reads: tuple[int, ...]         # slots bound to in0, in1, ...
    writes: tuple[int, ...]        # slots of out0, out1, ...


@dataclass(frozen=True)
class StageGraph:
    slot_names: tuple[str, ...]    # slot -> name (region inputs first)
    n_inputs: int
    nodes: tuple[StageNode, ...]
    outputs: tuple[int, ...]       # slot of each region output, in output order

    def walk_shapes(self, input_shapes, input_dtypes):
        """[(kernel, [(shape, dtype) per input], [shape per output])] per stage,
        and the (shape, dtype) of every region output."""
        from .kernels import _resolve_dtype

        meta: list = [None] * len(self.slot_names)
        for i, (s, d) in enumerate(zip(input_shapes, input_dtypes)):
            meta[i] = (tuple(s), d)
        walked = []
        for node in self.nodes:
            ins = [meta[i] for i in node.reads]
            env = [s for s, _ in ins]
            shapes = [tuple(int(Expr(e).evaluate(env)) for e in shp) for shp in node.kernel.output_shapes]
            dtypes = [_resolve_dtype(d, [dt for _, dt in ins]) for d in node.kernel.output_dtypes]
            for slot, s, d in zip(node.writes, shapes, dtypes):
                meta[slot] = (s, d)
            walked.append((node.kernel, ins, shapes))
        return walked, [meta[i] for i in self.outputs]


def _local_names(prefix: str, n: int) -> tuple[str, ...]:
    return tuple(f"{prefix}{j}" for j in range(n))


def _check_stage_kernel(i: int, stage) -> None:
    k = stage.kernel
    if k.stages:
        raise StageError("nested", i, f"kernel {k.kernel_id!r} has stages of its own")
    if k.fallback_predicate is not None or k.input_signature is not None or k.input_signatures is not None:
        raise StageError("stage_policy", i, f"kernel {k.kernel_id!r} carries a fallback or signature; "
                                            "put it on the region")
    if k.input_names != _local_names("in", len(stage.inputs)):
        raise StageError("local_inputs", i, f"kernel inputs {k.input_names} for {len(stage.inputs)} operands")
    if not stage.outputs or k.output_names != _local_names("out", len(stage.outputs)):
        raise StageError("local_outputs", i, f"kernel outputs {k.output_names} for results {stage.outputs}")
    if not len(k.output_shapes) == len(k.output_dtypes) == len(stage.outputs):
        raise StageError("out_meta", i, f"{len(stage.outputs)} results, {len(k.output_shapes)} shapes, "
                                        f"{len(k.output_dtypes)} dtypes")


def build_graph(spec) -> StageGraph:
    """Validate the spec's stages and return its dataflow graph."""
    names = list(spec.input_names)
    slot_of = {n: i for i, n in enumerate(names)}
    region_outs = set(spec.output_names)
    readers = [0] * len(names)
    nodes = []
    for i, stage in enumerate(spec.stages):
        _check_stage_kernel(i, stage)
        unbound = [x for x in stage.inputs if x not in slot_of]
        if unbound:
            raise StageError("unbound", i, f"reads {unbound} before anything produces them")
        reads = tuple(slot_of[x] for x in stage.inputs)
        for r in reads:
            readers[r] += 1
        writes = []
        for name in stage.outputs:
            if name in slot_of or not (name in region_outs or _TMP.fullmatch(name)):
                raise StageError("rebind", i, f"result {name!r} is not a fresh tmpN or region output")
            slot_of[name] = len(names)
            names.append(name)
            readers.append(0)
            writes.append(slot_of[name])
        nodes.append(StageNode(stage.kernel, reads, tuple(writes)))
    missing = [o for o in spec.output_names if o not in slot_of or slot_of[o] < len(spec.input_names)]
    if missing:
        raise StageError("unproduced", None, f"no stage produces {missing}")
    dead = [names[s] for s in range(len(spec.input_names), len(names))
            if readers[s] == 0 and names[s] not in region_outs]
    if dead:
        raise StageError("dead", None, f"{dead} are produced and never read; drop that work")
    return StageGraph(tuple(names), len(spec.input_names), tuple(nodes),
                      tuple(slot_of[o] for o in spec.output_names))


def wiring(spec):
    """(input slots of each stage, slot of each region output)."""
    g = build_graph(spec)
    return [n.reads for n in g.nodes], g.outputs


def shapes(spec, input_shapes, input_dtypes):
    """Stage-by-stage shapes and the region outputs' (shape, dtype)."""
    return build_graph(spec).walk_shapes(input_shapes, input_dtypes)
