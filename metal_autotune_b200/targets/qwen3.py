"""Qwen3 decoder (the Qwen3-4B-4bit target of models/qwen3_4b_4bit.py) as a
torch module tree with MLX-affine quantised projections, random-initialised.

The module forward methods are the *original op sequence*: plain torch ops in
the order and rounding of mlx-lm 0.31.3's qwen3 model (each op rounds to
bf16, projections dequantise with MLX rounding then matmul). They are what
the region wrappers of the bundle (bundles/qwen3_4b) replace, and what a
wrapper falls back to when a region's fallback predicate fires
(autotuner_runtime/kernels.py:254-268 semantics). Layer structure per
BASELINE configs[2] / the reference's model call: rms_norm -> q/k/v qmm ->
q_norm/k_norm -> rope(offset) -> causal GQA SDPA -> o qmm -> +residual ->
rms_norm -> gate/up qmm -> swiglu -> down qmm -> +residual; final norm;
tied lm_head on the quantised embedding.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import workload


@dataclass(frozen=True)
class Qwen3Config:
    hidden: int = 2560
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 9728
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    group: int = 64
    bits: int = 4
    max_len: int = 160  # KV-cache rows per layer (prefill 128 + decode)


QWEN3_4B = Qwen3Config()
TINY = Qwen3Config(hidden=512, layers=2, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)


class QLinear(nn.Module):
    """mlx.nn.QuantizedLinear layout: weight int32 [N, K*bits/32], scales/biases [N, K/group]."""

    def __init__(self, wq, scales, biases, group, bits):
        super().__init__()
        self.register_buffer("weight", wq)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group, self.bits = group, bits

    def forward(self, x):
        w = workload.dequantize(self.weight, self.scales, self.biases, self.group, self.bits)
        return torch.matmul(x, w.t())


class RMSNorm(nn.Module):
    def __init__(self, dim, eps, dtype, device):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype, device=device), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (xf * r * self.weight.float()).to(x.dtype)


class LayerCache:
    """One layer's KV cache: k/v [Hkv, cap, D] and the number of valid rows."""

    def __init__(self, kv_heads, cap, head_dim, dtype, device):
        self.k = torch.zeros(kv_heads, cap, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros(kv_heads, cap, head_dim, dtype=dtype, device=device)
        self.offset = 0


class KVCache:
    def __init__(self, cfg: Qwen3Config, dtype=torch.bfloat16, device="cuda"):
        self.layers = [LayerCache(cfg.kv_heads, cfg.max_len, cfg.head_dim, dtype, device) for _ in range(cfg.layers)]

    def reset(self):
        for c in self.layers:
            c.offset = 0


def _rope(x, offset, base):
    """x [H, T, D] (non-traditional, dims = D, scale 1)."""
    H, T, D = x.shape
    half = D // 2
    inv = torch.tensor([base ** (-2.0 * j / D) for j in range(half)], dtype=torch.float32, device=x.device)
    pos = torch.arange(offset, offset + T, device=x.device, dtype=torch.float32)
    th = pos[:, None] * inv[None, :]
    c, s = torch.cos(th), torch.sin(th)
    xf = x.float()
    a, b = xf[..., :half], xf[..., half:]
    return torch.cat([a * c - b * s, a * s + b * c], dim=-1).to(x.dtype)


class Attention(nn.Module):
    def __init__(self, cfg: Qwen3Config, projs, dtype, device):
        super().__init__()
        self.cfg = cfg
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = projs
        self.q_norm = RMSNorm(cfg.head_dim, cfg.eps, dtype, device)
        self.k_norm = RMSNorm(cfg.head_dim, cfg.eps, dtype, device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    def qkv(self, x):
        return self.q_proj(x), self.k_proj(x), self.v_proj(x)

    def prologue(self, q, k, v, cache: LayerCache):
        cfg = self.cfg
        T = q.shape[0]
        qh = self.q_norm(q.view(T, cfg.heads, cfg.head_dim)).transpose(0, 1)
        kh = self.k_norm(k.view(T, cfg.kv_heads, cfg.head_dim)).transpose(0, 1)
        vh = v.view(T, cfg.kv_heads, cfg.head_dim).transpose(0, 1)
        off = cache.offset
        qh = _rope(qh, off, cfg.rope_theta)
        kh = _rope(kh, off, cfg.rope_theta)
        cache.k[:, off:off + T] = kh
        cache.v[:, off:off + T] = vh
        return qh.contiguous()

    def attend(self, qh, cache: LayerCache, kv_len: int):
        cfg = self.cfg
        T = qh.shape[1]
        k = cache.k[:, :kv_len].repeat_interleave(cfg.heads // cfg.kv_heads, dim=0)
        v = cache.v[:, :kv_len].repeat_interleave(cfg.heads // cfg.kv_heads, dim=0)
        s = torch.matmul(qh.float(), k.float().transpose(1, 2)) * self.scale
        q_pos = torch.arange(kv_len - T, kv_len, device=qh.device)[:, None]
        k_pos = torch.arange(kv_len, device=qh.device)[None, :]
        s = s.masked_fill(k_pos > q_pos, float("-inf"))
        o = torch.matmul(torch.softmax(s, dim=-1), v.float()).to(qh.dtype)
        return o.transpose(0, 1).reshape(T, cfg.heads * cfg.head_dim)

    def forward(self, x, cache: LayerCache):
        q, k, v = self.qkv(x)
        qh = self.prologue(q, k, v, cache)
        o = self.attend(qh, cache, cache.offset + x.shape[0])
        return self.o_proj(o)


class MLP(nn.Module):
    def __init__(self, projs):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = projs

    def gate_up(self, x):
        return _swiglu(self.gate_proj(x), self.up_proj(x))

    def forward(self, x):
        return self.down_proj(self.gate_up(x))


def _swiglu(g, u):
    """silu(g) * u with each op rounded: sigmoid, g*sigmoid, *u."""
    sg = torch.sigmoid(g.float()).to(g.dtype)
    return (g * sg) * u


class DecoderLayer(nn.Module):
    def __init__(self, cfg, attn, mlp, dtype, device):
        super().__init__()
        self.self_attn = attn
        self.mlp = mlp
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.eps, dtype, device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.eps, dtype, device)

    def forward(self, h, cache: LayerCache):
        """h [T, hidden] -> [T, hidden]; advances nothing (the model advances offsets)."""
        a = self.self_attn(self.input_layernorm(h), cache)
        h = h + a
        return h + self.mlp(self.post_attention_layernorm(h))


class QEmbedding(nn.Module):
    def __init__(self, wq, scales, biases, group, bits):
        super().__init__()
        self.register_buffer("weight", wq)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.group, self.bits = group, bits

    def forward(self, tokens):
        w = self.weight[tokens.long()]
        return workload.dequantize(w, self.scales[tokens.long()], self.biases[tokens.long()], self.group, self.bits)

    def as_linear(self, x):
        w = workload.dequantize(self.weight, self.scales, self.biases, self.group, self.bits)
        return torch.matmul(x, w.t())


class Qwen3Model(nn.Module):
    def __init__(self, cfg: Qwen3Config, embed: QEmbedding, layers: list[DecoderLayer], dtype, device):
        super().__init__()
        self.cfg = cfg
        self.embed_tokens = embed
        self.layers = nn.ModuleList(layers)
        self.norm = RMSNorm(cfg.hidden, cfg.eps, dtype, device)

    def forward(self, tokens, cache: KVCache):
        """tokens int32 [T] -> (token int32 [1], logprob float32 [1]) for the
        last position, as mlx-lm generate_step picks (argmax of logprobs)."""
        T = tokens.shape[0]
        h = self.embed_tokens(tokens)
        for layer, c in zip(self.layers, cache.layers):
            h = layer(h, c)
        for c in cache.layers:
            c.offset += T
        last = self.norm(h[-1:])
        logits = self.embed_tokens.as_linear(last)
        self.last_logits = logits  # the last position's logits, for checks
        lse = torch.logsumexp(logits.float(), dim=-1, keepdim=True)
        lp = (logits.float() - lse.to(logits.dtype).float()).to(logits.dtype)
        tok = torch.argmax(lp, dim=-1).to(torch.int32)
        return tok, lp.float().gather(-1, tok.long()[:, None]).reshape(1)


def build(cfg: Qwen3Config = QWEN3_4B, seed: int = 0, device="cuda", dtype=torch.bfloat16) -> Qwen3Model:
    """Random-init Qwen3 with N(0, 0.02) weights quantised to MLX affine
    (group cfg.group, cfg.bits), norms = 1, generated on the device."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = lambda n, k: QLinear(*workload.random_quantized(n, k, group=cfg.group, bits=cfg.bits, dtype=dtype,
                                                        generator=g, device=device), cfg.group, cfg.bits)
    layers = []
    for _ in range(cfg.layers):
        attn = Attention(cfg, (q(cfg.heads * cfg.head_dim, cfg.hidden), q(cfg.kv_heads * cfg.head_dim, cfg.hidden),
                               q(cfg.kv_heads * cfg.head_dim, cfg.hidden), q(cfg.hidden, cfg.heads * cfg.head_dim)),
                         dtype, device)
        mlp = MLP((q(cfg.ffn, cfg.hidden), q(cfg.ffn, cfg.hidden), q(cfg.hidden, cfg.ffn)))
        layers.append(DecoderLayer(cfg, attn, mlp, dtype, device))
    embed = QEmbedding(*workload.random_quantized(cfg.vocab, cfg.hidden, group=cfg.group, bits=cfg.bits,
                                                  dtype=dtype, generator=g, device=device), cfg.group, cfg.bits)
    return Qwen3Model(cfg, embed, layers, dtype, device)


def request(model, tokens: torch.Tensor, cache: KVCache):
    """The benchmark request: prefill the prompt (all tokens at once from an
    empty cache), then one decode step on the picked token. Returns
    (prefill token, decode token, decode logprob), all on the device."""
    cache.reset()
    t0, _ = model(tokens, cache)
    t1, lp1 = model(t0, cache)
    return t0, t1, lp1
