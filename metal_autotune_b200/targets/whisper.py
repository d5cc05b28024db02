"""Whisper-large-v3-turbo audio encoder (the target of the reference's
models/whisper_large_v3_turbo_encoder.py:8-12, mlx-whisper 0.4.3's
AudioEncoder) as a torch module tree in fp16, random-initialised.

The forward methods are the *original op sequence* with MLX's rounding: each
op computes in fp32 and rounds its result to fp16 (conv and linear sums in
fp32 with the bias added before the one rounding of an addmm; GELU, layer
norm and softmax in fp32 on the rounded inputs). They are what the region
wrappers of the bundle (bundles/whisper_turbo) replace, and what a wrapper
falls back to when a region's predicate fires.

  x = gelu(conv1(mel)); x = gelu(conv2(x))          # [B, 3000, 128] -> [B, 1500, 1280]
  x = x + positional_embedding                      # sinusoids(1500, 1280)
  per block (32): x = x + attn(attn_ln(x)); x = x + mlp2(gelu(mlp1(mlp_ln(x))))
  x = ln_post(x)
attn: q, k (no bias), v projections, softmax(q k^T / sqrt(d)) v over 20 heads
of 64, out projection. Weights and biases N(0, 0.02), LayerNorm gains 1 and
shifts 0; the mel input N(0, 1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class WhisperConfig:
    n_mels: int = 128
    n_ctx: int = 1500        # positions after the stride-2 conv (3000 input frames)
    n_state: int = 1280
    n_head: int = 20
    n_layer: int = 32
    eps: float = 1e-5

    @property
    def frames(self) -> int:
        return 2 * self.n_ctx

    @property
    def head_dim(self) -> int:
        return self.n_state // self.n_head


WHISPER_TURBO = WhisperConfig()
TINY = WhisperConfig(n_mels=128, n_ctx=200, n_state=256, n_head=4, n_layer=2)


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    """Whisper's sinusoidal positional table [length, channels]: sin then cos
    of position * exp(-log(max_timescale) * i / (channels/2 - 1))."""
    inc = math.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2, dtype=torch.float64))
    t = torch.arange(length, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.sin(t), torch.cos(t)], dim=1).to(torch.float32)


def _r(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float16)


# ---- each op's original sequence, shared by the modules below and by the
# graph bundles' region patterns (bundles/graph_wrappers.py)
def linear(x, w, b=None):
    """mlx.nn.Linear: y = round(x w^T + b) (one rounding, fp32 sums)."""
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return _r(y)


def conv1d(x, w, b, stride: int, padding: int):
    """mlx.nn.Conv1d on channels-last x [B, L, Cin], weight [Cout, K, Cin]:
    conv rounded, then + bias rounded."""
    y = F.conv1d(x.float().transpose(1, 2), w.float().permute(0, 2, 1), stride=stride,
                 padding=padding).transpose(1, 2)
    return _r(_r(y).float() + b.float())


def layer_norm(x, w, b, eps: float):
    return _r(F.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), eps))


def residual_add(x, y):
    """x + y of two fp16 tensors, rounded once."""
    return _r(x.float() + y.float())


def attend(q, k, v, n_head: int):
    """q, k, v [B, L, n_state] -> softmax(q k^T / sqrt(d)) v, heads concatenated."""
    B, L, S = q.shape
    d = S // n_head
    sh = lambda t: t.float().view(B, L, n_head, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(sh(q), sh(k), sh(v), scale=1.0 / math.sqrt(d))
    return _r(o.transpose(1, 2).reshape(B, L, S))


def conv_gelu(x, w, b, stride: int):
    """Region: a conv of the stem, then GELU."""
    return gelu(conv1d(x, w, b, stride, 1))


def linear_gelu(x, w, b):
    """Region: fc1, then GELU."""
    return gelu(linear(x, w, b))


def linear_residual(x, w, b, res):
    """Region: a projection (out or fc2) added to the residual stream."""
    return residual_add(res, linear(x, w, b))


class Linear(nn.Module):
    """mlx.nn.Linear: y = round(x w^T + b) (one rounding, fp32 sums)."""

    def __init__(self, w: torch.Tensor, b: torch.Tensor | None):
        super().__init__()
        self.register_buffer("weight", w)
        self.register_buffer("bias", b if b is not None else None)

    def forward(self, x):
        return linear(x, self.weight, self.bias)


class Conv1d(nn.Module):
    """mlx.nn.Conv1d on channels-last x [B, L, Cin], weight [Cout, K, Cin]:
    conv rounded, then + bias rounded."""

    def __init__(self, w: torch.Tensor, b: torch.Tensor, stride: int, padding: int):
        super().__init__()
        self.register_buffer("weight", w)
        self.register_buffer("bias", b)
        self.stride, self.padding = stride, padding

    def forward(self, x):
        return conv1d(x, self.weight, self.bias, self.stride, self.padding)


class LayerNorm(nn.Module):
    def __init__(self, dim: int, eps: float, device):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.float16, device=device), requires_grad=False)
        self.bias = nn.Parameter(torch.zeros(dim, dtype=torch.float16, device=device), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        return layer_norm(x, self.weight, self.bias, self.eps)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """mlx.nn.gelu (exact erf form) on fp16 values, evaluated in fp32, rounded."""
    xf = x.float()
    return _r(xf * (1 + torch.erf(xf / math.sqrt(2))) / 2)


class MultiHeadAttention(nn.Module):
    def __init__(self, cfg: WhisperConfig, q, k, v, o):
        super().__init__()
        self.cfg = cfg
        self.query, self.key, self.value, self.out = q, k, v, o

    def attend(self, q, k, v):
        """q, k, v [B, L, n_state] -> softmax(q k^T / sqrt(d)) v, heads concatenated."""
        return attend(q, k, v, self.cfg.n_head)

    def forward(self, x):
        return self.out(self.attend(self.query(x), self.key(x), self.value(x)))


class ResidualAttentionBlock(nn.Module):
    def __init__(self, cfg, attn, mlp1, mlp2, device):
        super().__init__()
        self.attn = attn
        self.attn_ln = LayerNorm(cfg.n_state, cfg.eps, device)
        self.mlp1, self.mlp2 = mlp1, mlp2
        self.mlp_ln = LayerNorm(cfg.n_state, cfg.eps, device)

    def forward(self, x):
        x = residual_add(x, self.attn(self.attn_ln(x)))
        return residual_add(x, self.mlp2(gelu(self.mlp1(self.mlp_ln(x)))))


class AudioEncoder(nn.Module):
    def __init__(self, cfg, conv1, conv2, blocks, device):
        super().__init__()
        self.cfg = cfg
        self.conv1, self.conv2 = conv1, conv2
        self.register_buffer("positional_embedding", sinusoids(cfg.n_ctx, cfg.n_state).to(torch.float16).to(device))
        self.blocks = nn.ModuleList(blocks)
        self.ln_post = LayerNorm(cfg.n_state, cfg.eps, device)

    def forward(self, mel):
        """mel [B, frames, n_mels] fp16 -> [B, n_ctx, n_state] fp16."""
        x = gelu(self.conv1(mel))
        x = gelu(self.conv2(x))
        x = residual_add(x, self.positional_embedding)
        for blk in self.blocks:
            x = blk(x)
        return self.ln_post(x)


def build(cfg: WhisperConfig = WHISPER_TURBO, seed: int = 0, device="cuda") -> AudioEncoder:
    """Random init: every weight and bias N(0, 0.02) in fp16, generated on the device."""
    g = torch.Generator(device=device).manual_seed(seed)
    rnd = lambda *shape: (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.float16)
    S = cfg.n_state
    conv1 = Conv1d(rnd(S, 3, cfg.n_mels), rnd(S), 1, 1)
    conv2 = Conv1d(rnd(S, 3, S), rnd(S), 2, 1)
    blocks = []
    for _ in range(cfg.n_layer):
        attn = MultiHeadAttention(cfg, Linear(rnd(S, S), rnd(S)), Linear(rnd(S, S), None), Linear(rnd(S, S), rnd(S)),
                                  Linear(rnd(S, S), rnd(S)))
        blocks.append(ResidualAttentionBlock(cfg, attn, Linear(rnd(4 * S, S), rnd(4 * S)),
                                             Linear(rnd(S, 4 * S), rnd(S)), device))
    return AudioEncoder(cfg, conv1, conv2, blocks, device)


def encoder_flops(cfg: WhisperConfig, batch: int) -> float:
    """Algorithmic FLOPs of one encoder forward: the two convs, per block the
    q/k/v/out projections, attention (QK^T and PV) and the MLP."""
    S, L = cfg.n_state, cfg.n_ctx
    conv = 2 * cfg.frames * S * 3 * cfg.n_mels + 2 * L * S * 3 * S
    block = 2 * L * 4 * S * S + 2 * 2 * L * L * S + 2 * L * 8 * S * S
    return batch * (conv + cfg.n_layer * block)
