"""Candidate regions of one trace (the reference's autotuner/regions/build.py:
singletons plus chains grown from anchors, views absorbed, barriers, the
matmul-like rule, a length cap).

A stretch is a run of consecutive recorded calls with its boundary: the
arrays it reads from outside (inputs) and the ones something after it, or
the step's result, still needs (outputs). Candidates:
  * every non-view, non-barrier call alone;
  * chains from each anchor (the first call after a barrier, a change of
    module scope, a call reading only weights) to the next barrier, every
    prefix that ends on a computing call, up to MAX_STRETCH_COMPUTE_OPS.
A chain stops before a matmul-like call that reads a value produced by
another matmul-like call in the chain: every element of the second needs
the whole first result, which one kernel launch without a grid-wide barrier
cannot provide (build.py:24-30).
Barriers (never inside a stretch): in-place writes (aten ops whose name ends
in "_"), calls whose outputs nobody reads.
"""
from __future__ import annotations

from dataclasses import dataclass

from .trace import Trace, TraceNode

VIEW_OPS = frozenset({
    "view", "_unsafe_view", "reshape", "_reshape_alias", "t", "transpose", "permute", "expand", "unsqueeze",
    "squeeze", "slice", "select", "alias", "as_strided", "detach", "split", "split_with_sizes", "unbind",
    "view_as", "expand_as", "flatten", "unflatten", "narrow", "movedim", "lift_fresh", "chunk",
})

MATMUL_LIKE = frozenset({
    "mm", "bmm", "addmm", "baddbmm", "matmul", "linear", "convolution", "_convolution", "conv1d", "conv2d",
    "scaled_dot_product_attention", "_scaled_dot_product_flash_attention",
    "_scaled_dot_product_efficient_attention", "_scaled_dot_product_cudnn_attention",
    "_scaled_dot_product_flash_attention_for_cpu", "_scaled_mm",
})

MAX_STRETCH_COMPUTE_OPS = 64


def base(op: str) -> str:
    """aten.mm.default -> mm."""
    parts = op.split(".")
    return parts[1] if len(parts) > 1 else op


def is_view(node: TraceNode) -> bool:
    return base(node.op) in VIEW_OPS


def is_matmul_like(node: TraceNode) -> bool:
    return base(node.op) in MATMUL_LIKE


def _is_barrier(node: TraceNode, trace: Trace) -> bool:
    b = base(node.op)
    return (b.endswith("_") and not b.startswith("_")) or node.seq in trace.dead


@dataclass(frozen=True)
class Stretch:
    workload: str
    start_seq: int
    end_seq: int           # inclusive
    input_ids: tuple
    output_ids: tuple
    scope_stack: tuple


def weight_like_ids(trace: Trace) -> frozenset:
    """Weights and every view taken of one (a Linear's transposed matrix is
    still a weight to the kernel that reads it)."""
    ids = set(trace.weights)
    for node in trace.nodes:
        if is_view(node) and node.in_arrays and all(a in ids for a in node.in_arrays):
            ids.update(node.out_arrays)
    return frozenset(ids)


def boundary(trace: Trace, start: int, end: int) -> Stretch:
    nodes = trace.nodes[start:end + 1]
    produced, inputs = set(), []
    for node in nodes:
        for a in node.in_arrays:
            if a not in produced and a not in inputs:
                inputs.append(a)
        produced.update(node.out_arrays)
    outs, step = [], set(trace.step_outputs)
    for node in nodes:
        for a in node.out_arrays:
            if (a in step or any(s > end for s in trace.liveness[a].consumed_by)) and a not in outs:
                outs.append(a)
    common = []
    for parts in zip(*(n.module_stack for n in nodes)):
        if all(p == parts[0] for p in parts):
            common.append(parts[0])
        else:
            break
    return Stretch(trace.workload, start, end, tuple(inputs), tuple(outs), tuple(common) or ("",))


def build_stretches(trace: Trace) -> list[Stretch]:
    n = len(trace.nodes)
    barrier = [_is_barrier(node, trace) for node in trace.nodes]
    weight_like = weight_like_ids(trace)
    anchors = set()
    for i, node in enumerate(trace.nodes):
        if barrier[i]:
            continue
        if (i == 0 or barrier[i - 1] or node.module_address != trace.nodes[i - 1].module_address
                or (node.in_arrays and all(a in weight_like for a in node.in_arrays))):
            anchors.add(i)
    stretches, seen = [], set()

    def add(a: int, b: int) -> None:
        if (a, b) not in seen:
            seen.add((a, b))
            stretches.append(boundary(trace, a, b))

    for i, node in enumerate(trace.nodes):
        if barrier[i] or is_view(node):
            continue
        if any(a in weight_like and a not in trace.weights for a in node.in_arrays):
            continue  # a lone op on a viewed weight: the chain from the view is the candidate
        add(i, i)
    for a in sorted(anchors):
        compute, downstream = 0, set()
        for j in range(a, n):
            node = trace.nodes[j]
            if barrier[j]:
                break
            reads_down = any(x in downstream for x in node.in_arrays)
            if is_matmul_like(node) and reads_down:
                break
            if is_matmul_like(node) or reads_down:
                downstream.update(node.out_arrays)
            if not is_view(node):
                compute += 1
                if compute > MAX_STRETCH_COMPUTE_OPS:
                    break
                if j > a:
                    add(a, j)
    return stretches
