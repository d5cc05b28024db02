"""TEST INFRASTRUCTURE — Mamba-1 prefill composed from the oracle's region
restatements (numpy front end of liboracle.so).

Only tests/ and bench.py's CPU leg use this module. The sequence is
mlx-lm 0.31.3's mamba model as the reference runs it
(models/mamba_370m.py:4-8): per layer x + out_proj(scan(...) * silu(z)) on
rms_norm(x), with in_proj, the depthwise causal conv + SiLU, x_proj split
into (delta, B, C), dt_proj with its bias, the selective scan from a zero
state (Gu & Dao 2023); embedding, norm_f and the tied lm_head on the last
position. Every op rounds to fp16, the scan state is fp32.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import ref as R

DT = "float16"


def _np(t):
    return t.detach().float().cpu().numpy()


@dataclass
class LayerWeights:
    norm: np.ndarray
    in_proj: np.ndarray
    conv_w: np.ndarray
    conv_b: np.ndarray
    x_proj: np.ndarray
    dt_proj: np.ndarray
    dt_bias: np.ndarray
    A: np.ndarray        # -exp(A_log), fp32
    D: np.ndarray
    out_proj: np.ndarray


@dataclass
class ModelWeights:
    embedding: np.ndarray
    layers: list
    norm_f: np.ndarray


def layer_weights(layer) -> LayerWeights:
    m = layer.mixer
    import torch
    A = (-torch.exp(m.A_log.float())).cpu().numpy()
    return LayerWeights(_np(layer.norm.weight), _np(m.in_proj), _np(m.conv_w), _np(m.conv_b), _np(m.x_proj),
                        _np(m.dt_proj), _np(m.dt_bias), A, _np(m.D), _np(m.out_proj))


def model_weights(model, n_layers: int | None = None) -> ModelWeights:
    layers = list(model.layers)[:n_layers] if n_layers is not None else list(model.layers)
    return ModelWeights(_np(model.embedding), [layer_weights(l) for l in layers], _np(model.norm_f.weight))


def layer(cfg, W: LayerWeights, x):
    """x [L, d_model] -> x + mixer(rms_norm(x))."""
    E, Rk, S = cfg.d_inner, cfg.dt_rank, cfg.d_state
    h = R.rms_norm(x, W.norm, cfg.eps, DT)
    xs = R.linear_lp(h, W.in_proj[:E], None, 0, DT)
    z = R.linear_lp(h, W.in_proj[E:], None, 0, DT)
    xc = R.causal_conv1d(xs, W.conv_w, W.conv_b, None, True, DT)
    delta = R.linear_lp(xc, W.x_proj[:Rk], None, 0, DT)
    B = R.linear_lp(xc, W.x_proj[Rk:Rk + S], None, 0, DT)
    C = R.linear_lp(xc, W.x_proj[Rk + S:], None, 0, DT)
    dt = R.linear_lp(delta, W.dt_proj, W.dt_bias, 0, DT)
    y = R.mamba_scan(xc, dt, None, W.A, B, C, W.D, z, None, DT)
    return R.add(R.linear_lp(y, W.out_proj, None, 0, DT), x, DT)


def prefill(cfg, M: ModelWeights, tokens):
    """tokens [L] -> (last-position logits [vocab], greedy token)."""
    x = M.embedding[np.asarray(tokens, np.int64)]
    for W in M.layers:
        x = layer(cfg, W, x)
    last = R.rms_norm(x[-1:], M.norm_f, cfg.eps, DT)
    logits = R.linear_lp(last, M.embedding, None, 0, DT).reshape(-1)
    tok, _, _ = R.logits_pick(logits, DT)
    return logits, int(tok)
