"""Mamba-370m (the reference's models/mamba_370m.py:4-8, mlx-lm 0.31.3's
mamba model) as a torch module tree in fp16, random-initialised, for the
prefill workload (models/workloads/mamba_370m_prefill_128.yaml; BASELINE
configs[1] asks for 512 prompt tokens).

The forward methods are the *original op sequence* with MLX's rounding: each
op computes in fp32 and rounds its result to fp16, the selective-scan state
in fp32. They are what the region wrappers of the bundle (bundles/mamba_370m)
replace, and what a wrapper falls back to.

  per layer (48): x = x + mixer(rms_norm(x))
  mixer: xz = in_proj(h); x, z = split(xz)
         x = silu(conv1d(x))                        # depthwise causal, width 4, bias
         delta, B, C = split(x_proj(x), [dt_rank, d_state, d_state])
         dt = softplus(dt_proj(delta))              # dt_proj has a bias
         h_t = exp(dt A) h_{t-1} + dt B_t x_t;  y_t = C_t h_t + D x_t   (A = -exp(A_log))
         out_proj(y * silu(z))
  embedding -> layers -> norm_f -> tied lm_head on the last position -> greedy pick
Weights and biases N(0, 0.02), A_log = log(1..d_state) per channel, D = 1,
norms 1.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class MambaConfig:
    d_model: int = 1024
    n_layer: int = 48
    d_inner: int = 2048
    d_state: int = 16
    d_conv: int = 4
    dt_rank: int = 64
    vocab: int = 50280
    eps: float = 1e-5


MAMBA_370M = MambaConfig()
TINY = MambaConfig(d_model=256, n_layer=2, d_inner=512, d_state=16, d_conv=4, dt_rank=16, vocab=1000)


def _r(x):
    return x.to(torch.float16)


def _linear(x, w, b=None):
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return _r(y)


class RMSNorm(nn.Module):
    def __init__(self, dim, eps, device):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.float16, device=device), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return _r(xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float())


def _silu_rounded(v):
    sg = _r(torch.sigmoid(v.float()))
    return _r(v.float() * sg.float())


class Mixer(nn.Module):
    def __init__(self, cfg: MambaConfig, rnd, device):
        super().__init__()
        self.cfg = cfg
        E, S = cfg.d_inner, cfg.d_state
        self.register_buffer("in_proj", rnd(2 * E, cfg.d_model))
        self.register_buffer("conv_w", rnd(E, cfg.d_conv))
        self.register_buffer("conv_b", rnd(E))
        self.register_buffer("x_proj", rnd(cfg.dt_rank + 2 * S, E))
        self.register_buffer("dt_proj", rnd(E, cfg.dt_rank))
        self.register_buffer("dt_bias", rnd(E))
        self.register_buffer("A_log", torch.log(torch.arange(1, S + 1, dtype=torch.float32, device=device)).repeat(E, 1))
        self.register_buffer("D", torch.ones(E, dtype=torch.float32, device=device))
        self.register_buffer("out_proj", rnd(cfg.d_model, E))

    def conv(self, x):
        """Depthwise causal conv (left zero context), + bias rounded, SiLU rounded."""
        W = self.cfg.d_conv
        xp = F.pad(x.float().t()[None], (W - 1, 0))
        y = F.conv1d(xp, self.conv_w.float()[:, None, :], groups=x.shape[1])[0].t()
        return _silu_rounded(_r(y + self.conv_b.float()))

    def scan(self, x, dt, B, C, z):
        A = -torch.exp(self.A_log)
        h = torch.zeros_like(A)
        ys = []
        for t in range(x.shape[0]):
            d = F.softplus(dt[t].float())
            h = torch.exp(d[:, None] * A) * h + (d[:, None] * B[t].float()[None, :]) * x[t].float()[:, None]
            yv = (h * C[t].float()[None, :]).sum(-1) + self.D * x[t].float()
            zv = z[t].float()
            ys.append(yv * (zv * torch.sigmoid(zv)))
        return _r(torch.stack(ys))

    def forward(self, h):
        cfg = self.cfg
        E, R_, S = cfg.d_inner, cfg.dt_rank, cfg.d_state
        xz = _linear(h, self.in_proj)
        x, z = xz[:, :E], xz[:, E:]
        x = self.conv(x)
        dbc = _linear(x, self.x_proj)
        delta, B, C = dbc[:, :R_], dbc[:, R_:R_ + S], dbc[:, R_ + S:]
        dt = _linear(delta, self.dt_proj, self.dt_bias)
        return _linear(self.scan(x, dt, B, C, z), self.out_proj)


class ResidualBlock(nn.Module):
    def __init__(self, cfg, rnd, device):
        super().__init__()
        self.mixer = Mixer(cfg, rnd, device)
        self.norm = RMSNorm(cfg.d_model, cfg.eps, device)

    def forward(self, x):
        return _r(self.mixer(self.norm(x)).float() + x.float())


class MambaModel(nn.Module):
    def __init__(self, cfg, rnd, device):
        super().__init__()
        self.cfg = cfg
        self.register_buffer("embedding", rnd(cfg.vocab, cfg.d_model))
        self.layers = nn.ModuleList([ResidualBlock(cfg, rnd, device) for _ in range(cfg.n_layer)])
        self.norm_f = RMSNorm(cfg.d_model, cfg.eps, device)

    def forward(self, tokens):
        """tokens int32 [L] -> (greedy token int32 [1], last-position logits [1, vocab])."""
        x = self.embedding[tokens.long()]
        for layer in self.layers:
            x = layer(x)
        last = self.norm_f(x[-1:])
        logits = _linear(last, self.embedding)
        lse = torch.logsumexp(logits.float(), dim=-1, keepdim=True)
        lp = (logits.float() - lse.to(logits.dtype).float()).to(logits.dtype)
        return torch.argmax(lp, dim=-1).to(torch.int32), logits


def build(cfg: MambaConfig = MAMBA_370M, seed: int = 0, device="cuda") -> MambaModel:
    g = torch.Generator(device=device).manual_seed(seed)
    rnd = lambda *shape: (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.float16)
    return MambaModel(cfg, rnd, device)


def prefill_flops(cfg: MambaConfig, L: int) -> float:
    """Algorithmic FLOPs of a prefill of L tokens: the projections, the
    depthwise conv, the scan (about 6 d_state FLOPs per channel and step) and
    the lm_head of the last position."""
    E, S = cfg.d_inner, cfg.d_state
    proj = 2 * L * (cfg.d_model * 2 * E + E * (cfg.dt_rank + 2 * S) + cfg.dt_rank * E + E * cfg.d_model)
    conv = 2 * L * E * cfg.d_conv
    scan = 6 * L * E * S
    return cfg.n_layer * (proj + conv + scan) + 2 * cfg.vocab * cfg.d_model
