"""TEST INFRASTRUCTURE — the mlx-whisper audio encoder composed from the
oracle's region restatements (numpy front end of liboracle.so).

Only tests/ and bench.py's CPU leg use this module. The sequence is
mlx-whisper 0.4.3's AudioEncoder as the reference runs it
(models/whisper_large_v3_turbo_encoder.py:8-12): gelu(conv1), gelu(conv2),
+ positional embedding, per block x + out(attn(attn_ln(x))) and
x + mlp2(gelu(mlp1(mlp_ln(x)))), ln_post; each op rounded to fp16, the
linears as mx.addmm (fp32 sums, the bias added before the one rounding).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import ref as R

DT = "float16"


def _np(t):
    return None if t is None else t.detach().float().cpu().numpy()


@dataclass
class BlockWeights:
    ln1_w: np.ndarray
    ln1_b: np.ndarray
    wq: np.ndarray
    bq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    bv: np.ndarray
    wo: np.ndarray
    bo: np.ndarray
    ln2_w: np.ndarray
    ln2_b: np.ndarray
    w1: np.ndarray
    b1: np.ndarray
    w2: np.ndarray
    b2: np.ndarray


@dataclass
class EncoderWeights:
    conv1_w: np.ndarray
    conv1_b: np.ndarray
    conv2_w: np.ndarray
    conv2_b: np.ndarray
    pos: np.ndarray
    blocks: list
    lnp_w: np.ndarray
    lnp_b: np.ndarray


def block_weights(blk) -> BlockWeights:
    a = blk.attn
    return BlockWeights(_np(blk.attn_ln.weight), _np(blk.attn_ln.bias), _np(a.query.weight), _np(a.query.bias),
                        _np(a.key.weight), _np(a.value.weight), _np(a.value.bias), _np(a.out.weight),
                        _np(a.out.bias), _np(blk.mlp_ln.weight), _np(blk.mlp_ln.bias), _np(blk.mlp1.weight),
                        _np(blk.mlp1.bias), _np(blk.mlp2.weight), _np(blk.mlp2.bias))


def encoder_weights(enc, n_blocks: int | None = None) -> EncoderWeights:
    blocks = list(enc.blocks)[:n_blocks] if n_blocks is not None else list(enc.blocks)
    return EncoderWeights(_np(enc.conv1.weight), _np(enc.conv1.bias), _np(enc.conv2.weight), _np(enc.conv2.bias),
                          _np(enc.positional_embedding), [block_weights(b) for b in blocks], _np(enc.ln_post.weight),
                          _np(enc.ln_post.bias))


def stem(cfg, W: EncoderWeights, mel):
    """mel [B, frames, n_mels] -> gelu(conv2(gelu(conv1(mel)))) + positional embedding."""
    x = R.conv1d(mel, W.conv1_w, W.conv1_b, 1, 1, 1, DT)
    x = R.conv1d(x, W.conv2_w, W.conv2_b, 2, 1, 1, DT)
    return R.add(x, W.pos[None], DT)


def block(cfg, W: BlockWeights, x):
    """One residual attention block on x [B, L, n_state]."""
    B, L, S = x.shape
    H, D = cfg.n_head, cfg.head_dim
    h = R.layer_norm(x, W.ln1_w, W.ln1_b, cfg.eps, DT)
    q = R.linear_lp(h, W.wq, W.bq, 0, DT)
    k = R.linear_lp(h, W.wk, None, 0, DT)
    v = R.linear_lp(h, W.wv, W.bv, 0, DT)
    hd = lambda t: np.ascontiguousarray(t.reshape(B, L, H, D).transpose(0, 2, 1, 3))
    o = R.sdpa(hd(q), hd(k), hd(v), 1.0 / math.sqrt(D), False, 0, DT)
    o = np.ascontiguousarray(o.transpose(0, 2, 1, 3)).reshape(B, L, S)
    x = R.add(x, R.linear_lp(o, W.wo, W.bo, 0, DT), DT)
    h = R.layer_norm(x, W.ln2_w, W.ln2_b, cfg.eps, DT)
    f = R.linear_lp(h, W.w1, W.b1, 1, DT)
    return R.add(x, R.linear_lp(f, W.w2, W.b2, 0, DT), DT)


def encoder(cfg, W: EncoderWeights, mel):
    x = stem(cfg, W, mel)
    for bw in W.blocks:
        x = block(cfg, bw, x)
    return R.layer_norm(x, W.lnp_w, W.lnp_b, cfg.eps, DT)
