"""TEST INFRASTRUCTURE — the Qwen3 request composed from the oracle's region
restatements (numpy front end of liboracle.so).

Only tests/ and bench.py's CPU legs use this module: as the checker of the
GPU request, and as the timed CPU implementation of the path. The layer is
the op sequence of mlx-lm 0.31.3's qwen3 model as the reference runs it
(models/qwen3_4b_4bit.py:4-8; regions per
examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/patch/wrappers.py:
38-106): rms_norm -> q/k/v quantized_matmul -> q/k RMSNorm -> rope(offset)
-> cache append -> causal GQA SDPA -> o_proj + residual -> rms_norm ->
gate/up -> swiglu -> down + residual; final norm on the last row, tied
quantised lm_head, greedy pick of the log-probabilities (mlx-lm
generate_step; autotuner_runtime/inference.py:140-147).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import ref as R


@dataclass
class QWeights:
    wq: np.ndarray      # uint32 [N, K*bits/32]
    scales: np.ndarray  # float32 [N, K/group] (bf16 values)
    biases: np.ndarray


@dataclass
class LayerWeights:
    in_norm: np.ndarray
    post_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    q: QWeights
    k: QWeights
    v: QWeights
    o: QWeights
    gate: QWeights
    up: QWeights
    down: QWeights


@dataclass
class ModelWeights:
    embed: QWeights
    norm: np.ndarray
    layers: list


def _np(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _q(lin) -> QWeights:
    return QWeights(lin.weight.detach().cpu().numpy().view(np.uint32), _np(lin.scales), _np(lin.biases))


def layer_weights(L) -> LayerWeights:
    """Host copies of one torch DecoderLayer of metal_autotune_b200.targets.qwen3."""
    a, m = L.self_attn, L.mlp
    return LayerWeights(_np(L.input_layernorm.weight), _np(L.post_attention_layernorm.weight),
                        _np(a.q_norm.weight), _np(a.k_norm.weight), _q(a.q_proj), _q(a.k_proj), _q(a.v_proj),
                        _q(a.o_proj), _q(m.gate_proj), _q(m.up_proj), _q(m.down_proj))


def model_weights(model) -> ModelWeights:
    """Host copies of a torch Qwen3Model (the unwrapped module tree)."""
    return ModelWeights(_q(model.embed_tokens), _np(model.norm.weight), [layer_weights(L) for L in model.layers])


def empty_cache(cfg):
    shape = (cfg.kv_heads, cfg.max_len, cfg.head_dim)
    return [(np.zeros(shape, np.float32), np.zeros(shape, np.float32)) for _ in range(cfg.layers)]


def layer(cfg, W: LayerWeights, h, kc, vc, offset):
    """One decoder layer on [T, hidden] bf16 values; appends to kc/vc in place."""
    T = h.shape[0]
    qm = lambda x, p: R.quantized_matmul(x, p.wq, p.scales, p.biases, cfg.group, cfg.bits)
    xn = R.rms_norm(h, W.in_norm, cfg.eps)
    q, k, v = qm(xn, W.q), qm(xn, W.k), qm(xn, W.v)
    qh, _, _ = R.qk_norm_rope_cache(q, k, v, W.q_norm, W.k_norm, cfg.eps, kc, vc, cfg.heads, cfg.kv_heads,
                                    offset, cfg.rope_theta)
    kv = offset + T
    o = R.sdpa(qh[None], kc[None, :, :kv], vc[None, :, :kv], 1 / math.sqrt(cfg.head_dim), True, offset)
    o = o[0].transpose(1, 0, 2).reshape(T, -1)
    h2 = R.add(qm(o, W.o), h)
    xn2 = R.rms_norm(h2, W.post_norm, cfg.eps)
    act = R.swiglu(qm(xn2, W.gate), qm(xn2, W.up))
    return R.add(qm(act, W.down), h2)


def forward(cfg, M: ModelWeights, tokens, cache, offset, keep_layer0=False):
    """tokens [T] -> (last-position logits [vocab], layer-0 output or None)."""
    E = M.embed
    h = R.quantized_embedding(np.asarray(tokens, np.int32), E.wq, E.scales, E.biases, cfg.group, cfg.bits)
    first = None
    for i, W in enumerate(M.layers):
        kc, vc = cache[i]
        h = layer(cfg, W, h, kc, vc, offset)
        if i == 0 and keep_layer0:
            first = h.copy()
    last = R.rms_norm(h[-1:], M.norm, cfg.eps)
    logits = R.quantized_matmul(last, E.wq, E.scales, E.biases, cfg.group, cfg.bits).reshape(-1)
    return logits, first


@dataclass
class RequestResult:
    prefill_logits: np.ndarray
    token0: int
    decode_logits: np.ndarray
    token1: int
    logprob1: float
    layer0_prefill: np.ndarray | None = None
    layer0_decode: np.ndarray | None = None


def request(cfg, M: ModelWeights, tokens, keep_layer0=False, force_token0: int | None = None) -> RequestResult:
    """Prefill `tokens` from an empty cache, pick, one decode step, pick.
    `force_token0` feeds a given token to the decode step (the GPU's pick),
    so both sides decode the same input even when a near-tie in the prefill
    logits could pick differently."""
    cache = empty_cache(cfg)
    T = len(tokens)
    lg0, l0p = forward(cfg, M, tokens, cache, 0, keep_layer0)
    t0, _, _ = R.logits_pick(lg0)
    fed = t0 if force_token0 is None else force_token0
    lg1, l0d = forward(cfg, M, np.array([fed], np.int32), cache, T, keep_layer0)
    t1, lp1, _ = R.logits_pick(lg1)
    return RequestResult(lg0, int(t0), lg1, int(t1), float(lp1), l0p, l0d)
