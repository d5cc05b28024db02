"""The tiny GELU-MLP target (the reference's examples/tiny_mlp.py:5-6 shape
family; BASELINE configs[0] fixes it as): x fp32 [32, 256] ~ N(0, 1);
Linear 256 -> 1024 (+ bias) -> GELU -> Linear 1024 -> 256 (+ bias).

Weights Kaiming-uniform (torch.nn.init.kaiming_uniform_ with a = 0, fan_in,
ReLU gain sqrt(2): bound sqrt(6 / fan_in)), biases 0, all drawn from one CPU
generator seeded with 0 in the order w1, w2, x. The forward is the original
op sequence in fp32: each output a sequential-k fused multiply-add sum plus
the bias, GELU in its exact erf form (mlx.nn.GELU's default).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn


@dataclass(frozen=True)
class TinyMLPConfig:
    batch: int = 32
    d_in: int = 256
    d_hidden: int = 1024
    seed: int = 0


TINY_MLP = TinyMLPConfig()


def linear(x, w, b):
    """One Linear's original op: x w^T + b."""
    return x @ w.t() + b


def gelu(h):
    """GELU in its exact erf form."""
    return h * (1 + torch.erf(h / math.sqrt(2))) / 2


def linear_gelu(x, w, b):
    """The first region's original ops: the first Linear, then GELU."""
    return gelu(linear(x, w, b))


class Linear(nn.Module):
    def __init__(self, w, b):
        super().__init__()
        self.register_buffer("weight", w)
        self.register_buffer("bias", b)

    def forward(self, x):
        return linear(x, self.weight, self.bias)


class TinyMLP(nn.Module):
    def __init__(self, l1: Linear, l2: Linear):
        super().__init__()
        self.l1, self.l2 = l1, l2

    def forward(self, x):
        return self.l2(gelu(self.l1(x)))


def kaiming_uniform(n_out: int, n_in: int, g: torch.Generator) -> torch.Tensor:
    bound = math.sqrt(6.0 / n_in)
    return (torch.rand(n_out, n_in, generator=g, dtype=torch.float32) * 2 - 1) * bound


def build(cfg: TinyMLPConfig = TINY_MLP, device="cuda"):
    """(model, x): the seeded weights and the seeded input, on `device`."""
    g = torch.Generator().manual_seed(cfg.seed)
    w1 = kaiming_uniform(cfg.d_hidden, cfg.d_in, g)
    w2 = kaiming_uniform(cfg.d_in, cfg.d_hidden, g)
    x = torch.randn(cfg.batch, cfg.d_in, generator=g, dtype=torch.float32)
    model = TinyMLP(Linear(w1.to(device), torch.zeros(cfg.d_hidden, device=device)),
                    Linear(w2.to(device), torch.zeros(cfg.d_in, device=device)))
    return model, x.to(device)


def flops(cfg: TinyMLPConfig = TINY_MLP) -> float:
    return 2 * cfg.batch * cfg.d_in * cfg.d_hidden * 2
