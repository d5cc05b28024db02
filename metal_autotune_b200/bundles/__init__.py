"""Region bundles (the reference's artifact layout, docs/artifacts.md:174-190:
kernels/<id>.launch.json + swap_table.json + patch/wrappers.py) for the
targets, and the generator that writes them.

`python -m metal_autotune_b200.bundles` rewrites the committed bundles.
"""
from __future__ import annotations

import json
import math
import shutil
from pathlib import Path

from ..autotuner_runtime.kernels import KernelSpec, write_spec

HERE = Path(__file__).resolve().parent
WRAPPERS = HERE / "qwen3_wrappers.py"

QMM_GROUP, QMM_BITS = 64, 4


def _ws(n_total: str, kind: int):
    return {"workspace": {"query": "mt_qmm_workspace_bytes",
                          "args": [{"expr": "in0.shape[0]"}, {"expr": n_total}, {"expr": "in0.shape[1]"},
                                   {"int": QMM_BITS}, {"int": kind}]}}


def qwen3_specs(eps: float = 1e-6, rope_theta: float = 1e6, head_dim: int = 128) -> list[KernelSpec]:
    """Shape-generic specs of every Qwen3 region (2-D [tokens, features] activations)."""
    S = []
    S.append(KernelSpec(
        kernel_id="rms_norm", name="mt_rms_norm", input_names=("in0", "in1"), output_names=("out0",),
        cuda={"symbol": "mt_rms_norm", "args": [
            {"in": 0}, {"in": 1}, {"float": eps}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]"),), output_dtypes=("in0",), reassociates=True))
    S.append(KernelSpec(
        kernel_id="qkv_qmm", name="mt_quantized_matmul_multi", input_names=tuple(f"in{i}" for i in range(10)),
        output_names=("out0", "out1", "out2"),
        cuda={"symbol": "mt_quantized_matmul_multi", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"in": 3}, {"out": 0}, {"expr": "in1.shape[0]"},
            {"in": 4}, {"in": 5}, {"in": 6}, {"out": 1}, {"expr": "in4.shape[0]"},
            {"in": 7}, {"in": 8}, {"in": 9}, {"out": 2}, {"expr": "in7.shape[0]"},
            {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"}, {"int": QMM_GROUP}, {"int": QMM_BITS},
            {"dtype": "in0"}, _ws("in1.shape[0] + in4.shape[0] + in7.shape[0]", 0), {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[0]"), ("in0.shape[0]", "in4.shape[0]"),
                       ("in0.shape[0]", "in7.shape[0]")),
        output_dtypes=("in0", "in0", "in0"), fallback_predicate="in0.shape[1] % 64 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="qk_norm_rope_cache", name="mt_qk_norm_rope_cache", input_names=tuple(f"in{i}" for i in range(7)),
        output_names=("out0",),
        cuda={"symbol": "mt_qk_norm_rope_cache", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"expr": "in0.shape[1]"}, {"expr": "in1.shape[1]"}, {"in": 3},
            {"in": 4}, {"float": eps}, {"out": 0}, {"in": 5}, {"in": 6}, {"expr": "in0.shape[0]"},
            {"expr": f"in0.shape[1] // {head_dim}"}, {"expr": f"in1.shape[1] // {head_dim}"}, {"int": head_dim},
            {"expr": "in5.shape[1]"}, {"scalar": "offset"}, {"float": rope_theta}, {"dtype": "in0"},
            {"stream": True}]},
        output_shapes=((f"in0.shape[1] // {head_dim}", "in0.shape[0]", str(head_dim)),), output_dtypes=("in0",),
        fallback_predicate=f"in0.shape[1] % {head_dim} != 0 or in5.shape[2] != {head_dim}", reassociates=True))
    S.append(KernelSpec(
        kernel_id="sdpa_causal_gqa", name="mt_sdpa", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_sdpa", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"int": 1}, {"expr": "in0.shape[0]"},
            {"expr": "in1.shape[0]"}, {"expr": "in0.shape[1]"}, {"scalar": "kv_len"}, {"expr": "in0.shape[2]"},
            {"float": 1.0 / math.sqrt(head_dim)}, {"int": 1}, {"scalar": "offset"},
            {"int": 0}, {"expr": "in0.shape[1] * in0.shape[2]"}, {"expr": "in0.shape[2]"},
            {"int": 0}, {"expr": "in1.shape[1] * in1.shape[2]"}, {"expr": "in1.shape[2]"},
            {"int": 0}, {"expr": "in2.shape[1] * in2.shape[2]"}, {"expr": "in2.shape[2]"},
            {"int": 0}, {"expr": "in0.shape[2]"}, {"expr": "in0.shape[0] * in0.shape[2]"},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[1]", "in0.shape[0] * in0.shape[2]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[2] != 128 and in0.shape[2] != 64", reassociates=True))
    # decode: the q/k-norm + rope + cache prologue and the attention as one cut
    S.append(KernelSpec(
        kernel_id="qk_norm_rope_sdpa_decode", name="mt_qk_norm_rope_sdpa_decode",
        input_names=tuple(f"in{i}" for i in range(7)), output_names=("out0",),
        cuda={"symbol": "mt_qk_norm_rope_sdpa_decode", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"expr": "in0.shape[1]"}, {"expr": "in1.shape[1]"}, {"in": 3},
            {"in": 4}, {"float": eps}, {"out": 0}, {"in": 5}, {"in": 6}, {"expr": "in0.shape[0]"},
            {"expr": f"in0.shape[1] // {head_dim}"}, {"expr": f"in1.shape[1] // {head_dim}"}, {"int": head_dim},
            {"expr": "in5.shape[1]"}, {"scalar": "offset"}, {"float": rope_theta},
            {"float": 1.0 / math.sqrt(head_dim)}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]"),), output_dtypes=("in0",),
        fallback_predicate=(f"in0.shape[0] > 4 or in0.shape[1] % {head_dim} != 0 or in5.shape[2] != {head_dim} or "
                            f"(in0.shape[1] // in1.shape[1]) * in0.shape[0] > 16"),
        reassociates=True))
    for kid in ("o_proj_residual", "down_proj_residual"):
        S.append(KernelSpec(
            kernel_id=kid, name="mt_quantized_matmul_residual", input_names=tuple(f"in{i}" for i in range(5)),
            output_names=("out0",),
            cuda={"symbol": "mt_quantized_matmul_residual", "args": [
                {"in": 0}, {"in": 1}, {"in": 2}, {"in": 3}, {"in": 4}, {"out": 0}, {"expr": "in0.shape[0]"},
                {"expr": "in1.shape[0]"}, {"expr": "in0.shape[1]"}, {"int": QMM_GROUP}, {"int": QMM_BITS},
                {"dtype": "in0"}, _ws("in1.shape[0]", 0), {"stream": True}]},
            output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",),
            fallback_predicate="in0.shape[1] % 64 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="gate_up_swiglu", name="mt_quantized_matmul_swiglu", input_names=tuple(f"in{i}" for i in range(7)),
        output_names=("out0",),
        cuda={"symbol": "mt_quantized_matmul_swiglu", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"in": 3}, {"in": 4}, {"in": 5}, {"in": 6}, {"out": 0},
            {"expr": "in0.shape[0]"}, {"expr": "in1.shape[0]"}, {"expr": "in0.shape[1]"}, {"int": QMM_GROUP},
            {"int": QMM_BITS}, {"dtype": "in0"}, _ws("2 * in1.shape[0]", 1), {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[1] % 64 != 0", reassociates=True))
    # decode cuts with the RMSNorm before the matmul fused in (M <= 4, the
    # streamed decode kernel's shapes); prefill takes rms_norm + the matmul
    dec = f"in0.shape[0] > 4 or in0.shape[1] % {8 * QMM_GROUP} != 0 or in0.shape[1] > 16384"
    S.append(KernelSpec(
        kernel_id="rms_norm_qkv_qmm", name="mt_rms_norm_quantized_matmul_multi",
        input_names=tuple(f"in{i}" for i in range(11)), output_names=("out0", "out1", "out2"),
        cuda={"symbol": "mt_rms_norm_quantized_matmul_multi", "args": [
            {"in": 0}, {"in": 1}, {"float": eps},
            {"in": 2}, {"in": 3}, {"in": 4}, {"out": 0}, {"expr": "in2.shape[0]"},
            {"in": 5}, {"in": 6}, {"in": 7}, {"out": 1}, {"expr": "in5.shape[0]"},
            {"in": 8}, {"in": 9}, {"in": 10}, {"out": 2}, {"expr": "in8.shape[0]"},
            {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"}, {"int": QMM_GROUP}, {"int": QMM_BITS},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in2.shape[0]"), ("in0.shape[0]", "in5.shape[0]"),
                       ("in0.shape[0]", "in8.shape[0]")),
        output_dtypes=("in0", "in0", "in0"), fallback_predicate=dec, reassociates=True))
    S.append(KernelSpec(
        kernel_id="rms_norm_gate_up_swiglu", name="mt_rms_norm_quantized_matmul_swiglu",
        input_names=tuple(f"in{i}" for i in range(8)), output_names=("out0",),
        cuda={"symbol": "mt_rms_norm_quantized_matmul_swiglu", "args": [
            {"in": 0}, {"in": 1}, {"float": eps}, {"in": 2}, {"in": 3}, {"in": 4}, {"in": 5}, {"in": 6}, {"in": 7},
            {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in2.shape[0]"}, {"expr": "in0.shape[1]"},
            {"int": QMM_GROUP}, {"int": QMM_BITS}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in2.shape[0]"),), output_dtypes=("in0",), fallback_predicate=dec,
        reassociates=True))
    S.append(KernelSpec(
        kernel_id="rms_norm_lm_head", name="mt_rms_norm_quantized_matmul_multi",
        input_names=("in0", "in1", "in2", "in3", "in4"), output_names=("out0",),
        cuda={"symbol": "mt_rms_norm_quantized_matmul_multi", "args": [
            {"in": 0}, {"in": 1}, {"float": eps},
            {"in": 2}, {"in": 3}, {"in": 4}, {"out": 0}, {"expr": "in2.shape[0]"},
            {"null": True}, {"null": True}, {"null": True}, {"null": True}, {"int": 0},
            {"null": True}, {"null": True}, {"null": True}, {"null": True}, {"int": 0},
            {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"}, {"int": QMM_GROUP}, {"int": QMM_BITS},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in2.shape[0]"),), output_dtypes=("in0",), fallback_predicate=dec,
        reassociates=True))
    S.append(KernelSpec(
        kernel_id="quantized_embedding", name="mt_quantized_embedding", input_names=("in0", "in1", "in2", "in3"),
        output_names=("out0",),
        cuda={"symbol": "mt_quantized_embedding", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"in": 3}, {"out": 0}, {"expr": "in0.shape[0]"},
            {"expr": "in1.shape[0]"}, {"expr": f"in1.shape[1] * {32 // QMM_BITS}"}, {"int": QMM_GROUP},
            {"int": QMM_BITS}, {"dtype": "in2"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", f"in1.shape[1] * {32 // QMM_BITS}"),), output_dtypes=("in2",)))
    S.append(KernelSpec(
        kernel_id="lm_head", name="mt_quantized_matmul", input_names=("in0", "in1", "in2", "in3"),
        output_names=("out0",),
        cuda={"symbol": "mt_quantized_matmul", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"in": 3}, {"out": 0}, {"expr": "in0.shape[0]"},
            {"expr": "in1.shape[0]"}, {"expr": "in0.shape[1]"}, {"int": QMM_GROUP}, {"int": QMM_BITS},
            {"dtype": "in0"}, _ws("in1.shape[0]", 0), {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[1] % 64 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="logits_pick", name="mt_logits_pick", input_names=("in0",),
        output_names=("out0", "out1", "out2"),
        cuda={"symbol": "mt_logits_pick", "args": [
            {"in": 0}, {"expr": "in0.shape[0] * in0.shape[1]"}, {"dtype": "in0"}, {"out": 0}, {"out": 1},
            {"out": 2}, {"stream": True}]},
        output_shapes=(("1",), ("1",), ("1",)), output_dtypes=("int32", "float32", "float32"),
        fallback_predicate="in0.shape[0] != 1"))
    return S


LAYER_KERNELS = ["rms_norm", "qkv_qmm", "qk_norm_rope_cache", "sdpa_causal_gqa", "o_proj_residual",
                 "gate_up_swiglu", "down_proj_residual", "rms_norm_qkv_qmm", "rms_norm_gate_up_swiglu",
                 "qk_norm_rope_sdpa_decode"]
ROOT_KERNELS = ["quantized_embedding", "rms_norm", "lm_head", "logits_pick", "rms_norm_lm_head"]


def whisper_specs(eps: float = 1e-5) -> list[KernelSpec]:
    """Shape-generic specs of the mlx-whisper encoder regions (fp16 or bf16,
    activations [batch, positions, features])."""
    rows = "in0.shape[0] * in0.shape[1]"
    S = []
    for kid, stride in (("conv1_gelu", 1), ("conv2_gelu", 2)):
        S.append(KernelSpec(
            kernel_id=kid, name="mt_conv1d", input_names=("in0", "in1", "in2"), output_names=("out0",),
            cuda={"symbol": "mt_conv1d", "args": [
                {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"},
                {"expr": "in0.shape[2]"}, {"expr": "in1.shape[0]"}, {"expr": "in1.shape[1]"}, {"int": stride},
                {"int": 1}, {"int": 1}, {"dtype": "in0"}, {"stream": True}]},
            output_shapes=(("in0.shape[0]", f"(in0.shape[1] + 2 - in1.shape[1]) // {stride} + 1", "in1.shape[0]"),),
            output_dtypes=("in0",), fallback_predicate="in0.shape[2] % 32 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="pos_add", name="mt_add", input_names=("in0", "in1"), output_names=("out0",),
        cuda={"symbol": "mt_add", "args": [
            {"in": 0}, {"in": 1}, {"out": 0}, {"expr": "in0.shape[0] * in0.shape[1] * in0.shape[2]"},
            {"expr": "in1.shape[0] * in1.shape[1]"}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]", "in0.shape[2]"),), output_dtypes=("in0",),
        fallback_predicate="in1.shape[0] != in0.shape[1] or in1.shape[1] != in0.shape[2]"))
    S.append(KernelSpec(
        kernel_id="layer_norm", name="mt_layer_norm", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_layer_norm", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"float": eps}, {"out": 0}, {"expr": rows}, {"expr": "in0.shape[2]"},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]", "in0.shape[2]"),), output_dtypes=("in0",),
        reassociates=True))
    S.append(KernelSpec(
        kernel_id="qkv_linear", name="mt_linear", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_linear", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": rows}, {"expr": "in1.shape[0]"},
            {"expr": "in0.shape[2]"}, {"int": 0}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[2] % 8 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="self_attention", name="mt_sdpa", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_sdpa", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in0.shape[2]"},
            {"expr": "in1.shape[2]"}, {"expr": "in0.shape[1]"}, {"expr": "in1.shape[1]"}, {"expr": "in0.shape[3]"},
            {"float": 0.125}, {"int": 0}, {"int": 0},
            {"stride": [0, 0]}, {"stride": [0, 2]}, {"stride": [0, 1]},
            {"stride": [1, 0]}, {"stride": [1, 2]}, {"stride": [1, 1]},
            {"stride": [2, 0]}, {"stride": [2, 2]}, {"stride": [2, 1]},
            {"expr": "in0.shape[1] * in0.shape[2] * in0.shape[3]"}, {"expr": "in0.shape[3]"},
            {"expr": "in0.shape[2] * in0.shape[3]"}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]", "in0.shape[2] * in0.shape[3]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[3] != 64", ensure_row_contiguous=False, reassociates=True))
    for kid in ("out_proj_residual", "fc2_residual"):
        S.append(KernelSpec(
            kernel_id=kid, name="mt_linear_residual", input_names=("in0", "in1", "in2", "in3"),
            output_names=("out0",),
            cuda={"symbol": "mt_linear_residual", "args": [
                {"in": 0}, {"in": 1}, {"in": 2}, {"in": 3}, {"out": 0}, {"expr": rows}, {"expr": "in1.shape[0]"},
                {"expr": "in0.shape[2]"}, {"dtype": "in0"}, {"stream": True}]},
            output_shapes=(("in0.shape[0]", "in0.shape[1]", "in1.shape[0]"),), output_dtypes=("in0",),
            fallback_predicate="in0.shape[2] % 8 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="fc1_gelu", name="mt_linear", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_linear", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": rows}, {"expr": "in1.shape[0]"},
            {"expr": "in0.shape[2]"}, {"int": 1}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[2] % 8 != 0", reassociates=True))
    return S


def mamba_specs(eps: float = 1e-5) -> list[KernelSpec]:
    """Shape-generic specs of the mlx-lm mamba regions (activations [tokens, features])."""
    S = []
    S.append(KernelSpec(
        kernel_id="rms_norm", name="mt_rms_norm", input_names=("in0", "in1"), output_names=("out0",),
        cuda={"symbol": "mt_rms_norm", "args": [
            {"in": 0}, {"in": 1}, {"float": eps}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]"),), output_dtypes=("in0",), reassociates=True))
    S.append(KernelSpec(
        kernel_id="linear", name="mt_linear", input_names=("in0", "in1"), output_names=("out0",),
        cuda={"symbol": "mt_linear", "args": [
            {"in": 0}, {"in": 1}, {"null": True}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in1.shape[0]"},
            {"expr": "in0.shape[1]"}, {"int": 0}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[1] % 8 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="linear_bias", name="mt_linear", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_linear", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in1.shape[0]"},
            {"expr": "in0.shape[1]"}, {"int": 0}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[1] % 8 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="causal_conv1d_silu", name="mt_causal_conv1d", input_names=("in0", "in1", "in2"),
        output_names=("out0",),
        cuda={"symbol": "mt_causal_conv1d", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"null": True}, {"out": 0}, {"expr": "in0.shape[0]"},
            {"expr": "in0.shape[1]"}, {"expr": "in1.shape[1]"}, {"int": 1}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]"),), output_dtypes=("in0",)))
    S.append(KernelSpec(
        kernel_id="selective_scan", name="mt_mamba_scan", input_names=tuple(f"in{i}" for i in range(7)),
        output_names=("out0",),
        cuda={"symbol": "mt_mamba_scan", "args": [
            {"in": 0}, {"in": 1}, {"null": True}, {"in": 2}, {"in": 3}, {"in": 4}, {"in": 5}, {"in": 6}, {"out": 0},
            {"null": True}, {"expr": "in0.shape[0]"}, {"expr": "in0.shape[1]"}, {"expr": "in2.shape[1]"},
            {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]"),), output_dtypes=("in0",), reassociates=True))
    S.append(KernelSpec(
        kernel_id="out_proj_residual", name="mt_linear_residual", input_names=("in0", "in1", "in2"),
        output_names=("out0",),
        cuda={"symbol": "mt_linear_residual", "args": [
            {"in": 0}, {"in": 1}, {"null": True}, {"in": 2}, {"out": 0}, {"expr": "in0.shape[0]"},
            {"expr": "in1.shape[0]"}, {"expr": "in0.shape[1]"}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",),
        fallback_predicate="in0.shape[1] % 8 != 0", reassociates=True))
    S.append(KernelSpec(
        kernel_id="embedding", name="mt_embedding", input_names=("in0", "in1"), output_names=("out0",),
        cuda={"symbol": "mt_embedding", "args": [
            {"in": 0}, {"in": 1}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in1.shape[0]"},
            {"expr": "in1.shape[1]"}, {"dtype": "in1"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in1.shape[1]"),), output_dtypes=("in1",)))
    S.append(KernelSpec(
        kernel_id="logits_pick", name="mt_logits_pick", input_names=("in0",),
        output_names=("out0", "out1", "out2"),
        cuda={"symbol": "mt_logits_pick", "args": [
            {"in": 0}, {"expr": "in0.shape[0] * in0.shape[1]"}, {"dtype": "in0"}, {"out": 0}, {"out": 1},
            {"out": 2}, {"stream": True}]},
        output_shapes=(("1",), ("1",), ("1",)), output_dtypes=("int32", "float32", "float32"),
        fallback_predicate="in0.shape[0] != 1"))
    return S


MAMBA_LAYER_KERNELS = ["rms_norm", "linear", "linear_bias", "causal_conv1d_silu", "selective_scan",
                       "out_proj_residual"]
MAMBA_ROOT_KERNELS = ["embedding", "rms_norm", "linear", "logits_pick"]


def write_mamba_bundle(directory: str | Path, n_layers: int) -> Path:
    table = [{"scope_path": f"layers.{i}", "wrapper_class": "W_mamba_layer", "kernel_ids": MAMBA_LAYER_KERNELS}
             for i in range(n_layers)]
    table.append({"scope_path": "", "wrapper_class": "W_mamba_model", "kernel_ids": MAMBA_ROOT_KERNELS})
    full = n_layers == 48
    meta = {"target": "mamba", "layers": n_layers, **artifact_meta(
        "metal_autotune_b200.targets.mamba:build", "MAMBA_370M" if full else "TINY", 0, "mamba_prefill",
        {"prompt": {"seeded": {"kind": "randint", "shape": [512 if full else 64], "dtype": "int32", "seed": 0,
                               "high": 50280 if full else 1000}}},
        {"rtol": 2e-2, "atol": 2e-2}, steps=2 if full else 5)}
    return _write_bundle(Path(directory), mamba_specs(), table, HERE / "mamba_wrappers.py", meta)


def tiny_mlp_specs() -> list[KernelSpec]:
    """The two fp32 linears of the tiny GELU-MLP (mt_linear, act 1 / 0)."""
    S = []
    for kid, act in (("linear_gelu_f32", 1), ("linear_f32", 0)):
        S.append(KernelSpec(
            kernel_id=kid, name="mt_linear", input_names=("in0", "in1", "in2"), output_names=("out0",),
            cuda={"symbol": "mt_linear", "args": [
                {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": "in0.shape[0]"}, {"expr": "in1.shape[0]"},
                {"expr": "in0.shape[1]"}, {"int": act}, {"dtype": "in0"}, {"stream": True}]},
            output_shapes=(("in0.shape[0]", "in1.shape[0]"),), output_dtypes=("in0",)))
    return S


def write_tiny_mlp_bundle(directory: str | Path) -> Path:
    table = [{"scope_path": "", "wrapper_class": "W_tiny_mlp", "kernel_ids": ["linear_gelu_f32", "linear_f32"]}]
    d = Path(directory)
    (d / "workloads").mkdir(parents=True, exist_ok=True)
    from safetensors.torch import save_file

    from ..targets import tiny_mlp
    _, x = tiny_mlp.build(tiny_mlp.TINY_MLP, device="cpu")  # the BASELINE input (seed 0, after the weights)
    save_file({"i0": x.contiguous()}, str(d / "workloads" / "x.safetensors"))
    meta = {"target": "tiny_mlp", "layers": 2, **artifact_meta(
        "metal_autotune_b200.targets.tiny_mlp:build", "TINY_MLP", None, "tiny_mlp",
        {"x": {"file": "workloads/x.safetensors"}}, {"rtol": 1e-4, "atol": 1e-4}, steps=20)}
    return _write_bundle(d, tiny_mlp_specs(), table, HERE / "tiny_mlp_wrappers.py", meta)


WHISPER_BLOCK_KERNELS = ["layer_norm", "qkv_linear", "self_attention", "out_proj_residual", "fc1_gelu",
                         "fc2_residual"]
WHISPER_ROOT_KERNELS = ["conv1_gelu", "conv2_gelu", "pos_add", "layer_norm"]


def artifact_meta(builder: str, config: str | None, seed: int | None, entry: str, workloads: dict,
                  tolerances: dict | None, steps: int = 5) -> dict:
    """The bundle.json fields bundles/artifact.py reads to rebuild, check and
    time the target in a fresh process."""
    return {"builder": builder, "config": config, "seed": seed, "entry": entry, "workloads": workloads,
            "correctness_rule": "baseline_tolerance", "tolerances": tolerances,
            "final_benchmark": {"pairs": 4, "warmup_steps": 3, "steps": steps}}


def _write_bundle(d: Path, specs, table, wrappers: Path, meta: dict) -> Path:
    (d / "kernels").mkdir(parents=True, exist_ok=True)
    (d / "patch").mkdir(exist_ok=True)
    for spec in specs:
        write_spec(d / "kernels", spec)
    (d / "swap_table.json").write_text(json.dumps(table, indent=1) + "\n")
    shutil.copyfile(wrappers, d / "patch" / "wrappers.py")
    (d / "bundle.json").write_text(json.dumps(meta, indent=1) + "\n")
    return d


def write_whisper_bundle(directory: str | Path, n_layers: int) -> Path:
    table = [{"scope_path": f"blocks.{i}", "wrapper_class": "W_whisper_block", "kernel_ids": WHISPER_BLOCK_KERNELS}
             for i in range(n_layers)]
    table.append({"scope_path": "", "wrapper_class": "W_whisper_encoder", "kernel_ids": WHISPER_ROOT_KERNELS})
    full = n_layers == 32
    meta = {"target": "whisper_encoder", "layers": n_layers, **artifact_meta(
        "metal_autotune_b200.targets.whisper:build", "WHISPER_TURBO" if full else "TINY", 0, "whisper_encoder",
        {"mel": {"seeded": {"kind": "randn", "shape": [1, 3000, 128] if full else [2, 400, 128], "dtype": "float16",
                            "seed": 0}}},
        {"rtol": 2e-2, "atol": 4e-2}, steps=2 if full else 5)}
    return _write_bundle(Path(directory), whisper_specs(), table, HERE / "whisper_wrappers.py", meta)


def write_qwen3_bundle(directory: str | Path, n_layers: int) -> Path:
    d = Path(directory)
    (d / "kernels").mkdir(parents=True, exist_ok=True)
    (d / "patch").mkdir(exist_ok=True)
    for spec in qwen3_specs():
        write_spec(d / "kernels", spec)
    table = [{"scope_path": f"layers.{i}", "wrapper_class": "W_qwen3_layer", "kernel_ids": LAYER_KERNELS}
             for i in range(n_layers)]
    table.append({"scope_path": "", "wrapper_class": "W_qwen3_root", "kernel_ids": ROOT_KERNELS})
    (d / "swap_table.json").write_text(json.dumps(table, indent=1) + "\n")
    shutil.copyfile(WRAPPERS, d / "patch" / "wrappers.py")
    meta = {"target": "qwen3", "layers": n_layers, **artifact_meta(
        "metal_autotune_b200.targets.qwen3:build", "QWEN3_4B" if n_layers == 36 else "TINY", 0, "qwen3_prefill",
        {"prompt": {"seeded": {"kind": "randint", "shape": [128 if n_layers == 36 else 32], "dtype": "int32",
                               "seed": 0, "high": 151936 if n_layers == 36 else 1000}}},
        {"rtol": 5e-2, "atol": 5e-2})}
    (d / "bundle.json").write_text(json.dumps(meta, indent=1) + "\n")
    return d


# ------------------------------------------------------------------ graph-backend bundles
GRAPH_WRAPPERS = HERE / "graph_wrappers.py"
_TINY_MLP_MOD = "metal_autotune_b200.targets.tiny_mlp"
_WHISPER_MOD = "metal_autotune_b200.targets.whisper"


def tiny_mlp_graph_variants(batches=(32,)) -> dict:
    """The tiny MLP's graph rules per batch: the first linear + GELU, then
    the second linear (each one occurrence)."""
    from ..targets import tiny_mlp
    cfg = tiny_mlp.TINY_MLP
    D, H, f32 = cfg.d_in, cfg.d_hidden, "float32"
    out = []
    for B in batches:
        out.append({"args": [[[B, D], f32]], "rules": [
            {"kernel_id": "linear_gelu_f32", "sequence": f"{_TINY_MLP_MOD}:linear_gelu",
             "input_specs": [[[B, D], f32], [[H, D], f32], [[H], f32]], "count": 1},
            {"kernel_id": "linear_f32", "sequence": f"{_TINY_MLP_MOD}:linear",
             "input_specs": [[[B, H], f32], [[D, H], f32], [[D], f32]], "count": 1}]})
    return {"G_tiny_mlp": out}


def whisper_graph_specs(n_head: int, head_dim: int = 64) -> list[KernelSpec]:
    """Specs the graph rules add to the Whisper regions: self-attention on the
    [B, L, n_state] projections (heads split by strides), and the q/v and k
    projections as separate linears."""
    S = [s for s in whisper_specs() if s.kernel_id in
         ("conv1_gelu", "conv2_gelu", "pos_add", "fc1_gelu", "fc2_residual", "out_proj_residual", "layer_norm")]
    row = "in0.shape[1] * in0.shape[2]"
    S.append(KernelSpec(
        kernel_id="attention", name="mt_sdpa", input_names=("in0", "in1", "in2"), output_names=("out0",),
        cuda={"symbol": "mt_sdpa", "args": [
            {"in": 0}, {"in": 1}, {"in": 2}, {"out": 0}, {"expr": "in0.shape[0]"}, {"int": n_head}, {"int": n_head},
            {"expr": "in0.shape[1]"}, {"expr": "in1.shape[1]"}, {"int": head_dim},
            {"float": 1.0 / math.sqrt(head_dim)}, {"int": 0}, {"int": 0},
            {"expr": row}, {"int": head_dim}, {"expr": "in0.shape[2]"},
            {"expr": "in1.shape[1] * in1.shape[2]"}, {"int": head_dim}, {"expr": "in1.shape[2]"},
            {"expr": "in2.shape[1] * in2.shape[2]"}, {"int": head_dim}, {"expr": "in2.shape[2]"},
            {"expr": row}, {"int": head_dim}, {"expr": "in0.shape[2]"}, {"dtype": "in0"}, {"stream": True}]},
        output_shapes=(("in0.shape[0]", "in0.shape[1]", "in0.shape[2]"),), output_dtypes=("in0",),
        fallback_predicate=f"in0.shape[2] != {n_head * head_dim}", reassociates=True))
    rows = "in0.shape[0] * in0.shape[1]"
    for kid, bias in (("linear_bias", {"in": 2}), ("linear_nobias", {"null": True})):
        n_in = 3 if kid == "linear_bias" else 2
        S.append(KernelSpec(
            kernel_id=kid, name="mt_linear", input_names=tuple(f"in{i}" for i in range(n_in)), output_names=("out0",),
            cuda={"symbol": "mt_linear", "args": [
                {"in": 0}, {"in": 1}, bias, {"out": 0}, {"expr": rows}, {"expr": "in1.shape[0]"},
                {"expr": "in0.shape[2]"}, {"int": 0}, {"dtype": "in0"}, {"stream": True}]},
            output_shapes=(("in0.shape[0]", "in0.shape[1]", "in1.shape[0]"),), output_dtypes=("in0",),
            fallback_predicate="in0.shape[2] % 8 != 0", reassociates=True))
    return S


def whisper_graph_variants(cfg, batches) -> dict:
    """The encoder's graph rules per batch, larger regions first (a rule
    rewrites before the next one looks for its pattern)."""
    S, L, T, M, n, f16 = cfg.n_state, cfg.n_ctx, cfg.frames, cfg.n_mels, cfg.n_layer, "float16"
    out = []
    for B in batches:
        act = [[B, L, S], f16]
        vec = lambda k: [[k], f16]
        out.append({"args": [[[B, T, M], f16]], "rules": [
            {"kernel_id": "conv1_gelu", "sequence": f"{_WHISPER_MOD}:conv_gelu", "bind": {"stride": 1},
             "input_specs": [[[B, T, M], f16], [[S, 3, M], f16], vec(S)], "count": 1},
            {"kernel_id": "conv2_gelu", "sequence": f"{_WHISPER_MOD}:conv_gelu", "bind": {"stride": 2},
             "input_specs": [[[B, T, S], f16], [[S, 3, S], f16], vec(S)], "count": 1},
            {"kernel_id": "pos_add", "sequence": f"{_WHISPER_MOD}:residual_add",
             "input_specs": [act, [[L, S], f16]], "count": 1,
             "anchors": [None, ["weight", "positional_embedding"]]},
            {"kernel_id": "fc1_gelu", "sequence": f"{_WHISPER_MOD}:linear_gelu",
             "input_specs": [act, [[4 * S, S], f16], vec(4 * S)], "count": n},
            {"kernel_id": "fc2_residual", "sequence": f"{_WHISPER_MOD}:linear_residual",
             "input_specs": [[[B, L, 4 * S], f16], [[S, 4 * S], f16], vec(S), act], "count": n},
            {"kernel_id": "out_proj_residual", "sequence": f"{_WHISPER_MOD}:linear_residual",
             "input_specs": [act, [[S, S], f16], vec(S), act], "count": n},
            {"kernel_id": "attention", "sequence": f"{_WHISPER_MOD}:attend", "bind": {"n_head": cfg.n_head},
             "input_specs": [act, act, act], "count": n},
            {"kernel_id": "linear_bias", "sequence": f"{_WHISPER_MOD}:linear",
             "input_specs": [act, [[S, S], f16], vec(S)], "count": 2 * n},
            {"kernel_id": "linear_nobias", "sequence": f"{_WHISPER_MOD}:linear",
             "input_specs": [act, [[S, S], f16]], "count": n},
            {"kernel_id": "layer_norm", "sequence": f"{_WHISPER_MOD}:layer_norm", "bind": {"eps": cfg.eps},
             "input_specs": [act, vec(S), vec(S)], "count": 2 * n + 1}]})
    return {"G_whisper_encoder": out}


def _write_graph_bundle(d: Path, specs, wrapper_class: str, kernel_ids, variants: dict, meta: dict) -> Path:
    table = [{"scope_path": "", "wrapper_class": wrapper_class, "kernel_ids": list(kernel_ids)}]
    _write_bundle(d, specs, table, GRAPH_WRAPPERS, {**meta, "backend": "graph"})
    (d / "patch" / "graph_variants.json").write_text(json.dumps(variants, indent=1) + "\n")
    return d


def write_tiny_mlp_graph_bundle(directory: str | Path) -> Path:
    d = Path(directory)
    (d / "workloads").mkdir(parents=True, exist_ok=True)
    from safetensors.torch import save_file

    from ..targets import tiny_mlp
    _, x = tiny_mlp.build(tiny_mlp.TINY_MLP, device="cpu")  # the BASELINE input (seed 0, after the weights)
    save_file({"i0": x.contiguous()}, str(d / "workloads" / "x.safetensors"))
    meta = {"target": "tiny_mlp", "layers": 2, **artifact_meta(
        "metal_autotune_b200.targets.tiny_mlp:build", "TINY_MLP", None, "tiny_mlp",
        {"x": {"file": "workloads/x.safetensors"}}, {"rtol": 1e-4, "atol": 1e-4}, steps=20)}
    return _write_graph_bundle(d, tiny_mlp_specs(), "G_tiny_mlp", ["linear_gelu_f32", "linear_f32"],
                               tiny_mlp_graph_variants(), meta)


def write_whisper_graph_bundle(directory: str | Path, n_layers: int) -> Path:
    from ..targets import whisper
    cfg = whisper.WHISPER_TURBO if n_layers == 32 else whisper.TINY
    full = n_layers == 32
    batches = (1, 8) if full else (2,)
    meta = {"target": "whisper_encoder", "layers": n_layers, **artifact_meta(
        "metal_autotune_b200.targets.whisper:build", "WHISPER_TURBO" if full else "TINY", 0, "whisper_encoder",
        {"mel": {"seeded": {"kind": "randn", "shape": [1, 3000, 128] if full else [2, 400, 128], "dtype": "float16",
                            "seed": 0}}},
        {"rtol": 2e-2, "atol": 4e-2}, steps=2 if full else 5)}
    specs = whisper_graph_specs(cfg.n_head, cfg.head_dim)
    return _write_graph_bundle(Path(directory), specs, "G_whisper_encoder", [s.kernel_id for s in specs],
                               whisper_graph_variants(cfg, batches), meta)


BUNDLES = {
    "qwen3_4b": lambda d: write_qwen3_bundle(d, 36),
    "qwen3_tiny": lambda d: write_qwen3_bundle(d, 2),
    "whisper_turbo": lambda d: write_whisper_bundle(d, 32),
    "whisper_tiny": lambda d: write_whisper_bundle(d, 2),
    "mamba_370m": lambda d: write_mamba_bundle(d, 48),
    "mamba_tiny": lambda d: write_mamba_bundle(d, 2),
    "tiny_mlp": write_tiny_mlp_bundle,
    "tiny_mlp_graph": write_tiny_mlp_graph_bundle,
    "whisper_turbo_graph": lambda d: write_whisper_graph_bundle(d, 32),
    "whisper_tiny_graph": lambda d: write_whisper_graph_bundle(d, 2),
}


def main() -> None:
    for name, write in BUNDLES.items():
        write(HERE / name)


if __name__ == "__main__":
    main()
