"""Seeded synthetic inputs and MLX-affine quantised random weights.

Token inputs follow the reference's workload declarations (autotuner/
workload.py:31-69; models/workloads/qwen3_4b_prefill_128.yaml: shape [1,128],
int32 in [0, 151936)) with torch's seeded Philox generator in place of MLX's
RNG (which cannot be reproduced here); the seed is recorded by callers.

quantize_affine packs weights the way mlx.core.quantize lays them out (the
layout of autotuner/scaffold/lower.py:468-514): per group of `group` values
along K, scale = (max-min)/(2^bits-1), bias = min, q = round((w-bias)/scale)
clipped, scale/bias in the model dtype, q values packed into uint32 words
low-bits-first (held in int32 tensors: only the bits matter).
"""
from __future__ import annotations

import torch


def seeded_tokens(shape, low: int, high: int, seed: int = 0, device="cuda") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(low, high, tuple(shape), generator=g, dtype=torch.int64).to(torch.int32).to(device)


def pack(q: torch.Tensor, bits: int) -> torch.Tensor:
    """q [N, K] integer values < 2^bits -> int32 [N, K*bits/32] packed low-first."""
    N, K = q.shape
    per = 32 // bits
    shifts = (torch.arange(per, device=q.device, dtype=torch.int64) * bits)
    words = (q.to(torch.int64).reshape(N, K // per, per) << shifts).sum(dim=2)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words)
    return words.to(torch.int32).contiguous()


def unpack(wq: torch.Tensor, bits: int) -> torch.Tensor:
    per = 32 // bits
    w64 = wq.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, device=wq.device, dtype=torch.int64) * bits
    return ((w64[:, :, None] >> shifts) & ((1 << bits) - 1)).reshape(wq.shape[0], -1)


def quantize_affine(w: torch.Tensor, group: int = 64, bits: int = 4, dtype=torch.bfloat16):
    """w [N, K] float -> (int32 packed [N, K*bits/32], scales [N, K/group], biases [N, K/group])."""
    N, K = w.shape
    levels = (1 << bits) - 1
    g = w.float().reshape(N, K // group, group)
    lo = g.amin(dim=2)
    hi = g.amax(dim=2)
    scale = torch.clamp((hi - lo) / levels, min=1e-8).to(dtype)
    bias = lo.to(dtype)
    q = torch.clamp(torch.round((g - bias.float()[..., None]) / scale.float()[..., None]), 0, levels)
    return pack(q.reshape(N, K).to(torch.int32), bits), scale.contiguous(), bias.contiguous()


def dequantize(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group: int = 64, bits: int = 4):
    """MLX rounding: round(round(s*q) + b) in the scales' dtype (used by the
    unpatched torch model)."""
    q = unpack(wq, bits)
    N, K = q.shape
    s = scales.repeat_interleave(group, dim=1)
    b = biases.repeat_interleave(group, dim=1)
    return (s * q.to(scales.dtype)) + b  # each torch op rounds to the dtype


def random_quantized(N: int, K: int, *, group=64, bits=4, std=0.02, dtype=torch.bfloat16, generator=None,
                     device="cuda", chunk_rows=16384):
    """N(0, std) weights quantised to MLX affine, generated on the device in row chunks."""
    outs_w, outs_s, outs_b = [], [], []
    for r0 in range(0, N, chunk_rows):
        n = min(chunk_rows, N - r0)
        w = torch.randn(n, K, device=device, dtype=torch.float32, generator=generator) * std
        w = w.to(dtype)
        wq, s, b = quantize_affine(w, group, bits, dtype)
        outs_w.append(wq)
        outs_s.append(s)
        outs_b.append(b)
    return torch.cat(outs_w), torch.cat(outs_s), torch.cat(outs_b)
