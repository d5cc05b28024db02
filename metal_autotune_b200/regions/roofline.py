"""A region's physical limit on a B200 (the reference's
autotuner/regions/roofline.py): bytes crossing the region's boundary over
the measured HBM bandwidth, estimated FLOPs over the tensor (16-bit) or FMA
(fp32) rate, and one launch; the largest is the roofline, and
s_max = measured time / roofline is the most an ideal kernel could gain.

Peaks: MEASURED_PEAKS.json (the driver's STREAM-style copy and cuBLAS bf16
GEMM on this pool) when present, else the pool's earlier measurement
(6.65 TB/s, 1.59 PFLOP/s). fp32 arithmetic is priced at the B200's nominal
non-tensor FMA rate, 148 SMs x 128 lanes x 2 FLOP x 1.965 GHz = 74.4
TFLOP/s; a launch at LAUNCH_US.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass
from pathlib import Path

from .build import Stretch, base, is_view
from .trace import Trace, TraceNode

LAUNCH_US = 2.0
FP32_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12

_BYTES = {"bool": 1, "uint8": 1, "int8": 1, "int16": 2, "float16": 2, "bfloat16": 2, "int32": 4, "float32": 4,
          "uint32": 4, "int64": 8, "float64": 8}


@dataclass(frozen=True)
class Peaks:
    hbm_gbs: float
    tflops: dict         # dtype -> TFLOP/s
    launch_us: float
    source: str


def peaks() -> Peaks:
    f = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        hbm, tc, src = float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    else:
        hbm, tc, src = 6650.0, 1590.0, "fallback"
    return Peaks(hbm, {"bfloat16": tc, "float16": tc, "float32": FP32_TFLOPS}, LAUNCH_US, src)


def _numel(shape) -> int:
    return math.prod(shape)


def spec_bytes(spec) -> int:
    shape, dtype = spec
    return _numel(shape) * _BYTES.get(dtype, 4)


def node_flops(node: TraceNode) -> float:
    """FLOPs estimated from op and shapes: 2*M*N*K for products, 2 per
    output element per weight element of a convolution, 4*numel(q)*Lk for
    attention, a few per element for norms and softmax, one otherwise."""
    b = base(node.op)
    out = sum(_numel(s) for s, _ in node.out_specs)
    if is_view(node):
        return 0.0
    if b in ("mm", "bmm", "matmul"):
        return 2.0 * out * node.in_specs[0][0][-1]
    if b in ("addmm", "baddbmm"):
        return 2.0 * out * node.in_specs[1][0][-1]
    if b in ("convolution", "_convolution", "conv1d", "conv2d"):
        return 2.0 * out * _numel(node.in_specs[1][0][1:])
    if "scaled_dot_product" in b:
        q, k = node.in_specs[0][0], node.in_specs[1][0]
        return 4.0 * _numel(q) * k[-2]
    if b in ("native_layer_norm", "layer_norm", "rms_norm", "_fused_rms_norm"):
        return 4.0 * _numel(node.out_specs[0][0])
    if b in ("_softmax", "softmax", "_log_softmax", "log_softmax", "logsumexp"):
        return 5.0 * out
    if b in ("sum", "mean", "amax", "max", "min", "var", "std", "prod"):
        return float(sum(_numel(s) for s, _ in node.in_specs))
    return float(out)


def _dtype(node: TraceNode) -> str:
    return next((d for _, d in node.out_specs if d in ("float16", "bfloat16", "float32")), "float32")


def compute_ms(nodes, pk: Peaks) -> float:
    return sum(node_flops(n) / (pk.tflops.get(_dtype(n), FP32_TFLOPS) * 1e9) for n in nodes)


@dataclass(frozen=True)
class Roofline:
    t_mem_ms: float
    t_compute_ms: float
    t_launch_ms: float
    t_roofline_ms: float
    bound: str           # memory | compute | launch
    s_max: float


def stretch_roofline(trace: Trace, s: Stretch, pk: Peaks, t_orig_ms: float = 0.0) -> Roofline:
    nodes = trace.nodes[s.start_seq:s.end_seq + 1]
    nbytes = sum(spec_bytes(trace.specs[a]) for a in s.input_ids + s.output_ids)
    t_mem = nbytes / (pk.hbm_gbs * 1e9) * 1e3
    t_c = compute_ms(nodes, pk)
    t_l = pk.launch_us / 1e3
    t = max(t_mem, t_c, t_l)
    bound = "memory" if t == t_mem else "compute" if t == t_c else "launch"
    return Roofline(t_mem, t_c, t_l, t, bound, (t_orig_ms / t) if t > 0 and t_orig_ms > 0 else 1.0)


def step_floor(trace: Trace, pk: Peaks, step_ms: float) -> dict:
    """The whole step against its physics: bytes from outside it (weights,
    inputs) plus its outputs, every recorded op's FLOPs, the launches the
    eager step fires (roofline.py:118-150)."""
    produced, outside, launches = set(), {}, 0
    for node in trace.nodes:
        if node.seq in trace.dead:
            continue
        for a in node.in_arrays:
            if a not in produced:
                outside.setdefault(a, spec_bytes(trace.specs[a]))
        produced.update(node.out_arrays)
        launches += not is_view(node)
    total = sum(outside.values()) + sum(spec_bytes(trace.specs[a]) for a in trace.step_outputs)
    t_mem = total / (pk.hbm_gbs * 1e9) * 1e3
    t_c = compute_ms([n for n in trace.nodes if n.seq not in trace.dead], pk)
    floor = max(t_mem, t_c)
    return {"bytes_mb": total / 1e6, "gflop": sum(node_flops(n) for n in trace.nodes) / 1e9, "launches": launches,
            "t_mem_ms": t_mem, "t_compute_ms": t_c, "floor_ms": floor, "step_ms": step_ms,
            "room": (1.0 - floor / step_ms) if step_ms > 0 else None}
