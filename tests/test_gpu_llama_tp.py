"""Llama tensor-parallel forward on one B200 (small config, 8-bit affine).

tp = 1 is checked against a plain fp32 torch restatement of the same layer
sequence on the dequantised weights (every op of the CUDA path rounds to
bf16, the restatement does not: relative-norm tolerance below); tp = 2 and
tp = 4, with all shards in this process and the partial sums added in shard
order, are checked against tp = 1, which they match up to the rounding of
each shard's partial to bf16 before the sum; at 384 tokens (the fused
quantized matmul) and at 1024 (weights dequantised once, tcgen05 GEMM)."""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from metal_autotune_b200 import lib, workload
from metal_autotune_b200.targets import llama_tp

pytestmark = pytest.mark.gpu

CFG = llama_tp.LlamaConfig(hidden=512, layers=2, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=1024)
REL_TOL = 3e-2  # ||ours - ref|| / ||ref|| over the logits, bf16 activations vs fp32


def _tokens(B, L):
    return workload.seeded_tokens((B, L), 0, CFG.vocab, seed=3)


def _restated(m: llama_tp.LlamaTP, tokens):
    cfg = m.cfg
    (sh,) = m.shards
    deq = lambda s: workload.dequantize(*s, cfg.group, cfg.bits).float()
    B, L = tokens.shape
    D = cfg.head_dim
    rms = lambda x: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.eps)
    inv = cfg.rope_theta ** (-torch.arange(0, D // 2, device="cuda").float() * 2 / D)
    ang = torch.arange(L, device="cuda").float()[:, None] * inv[None]
    cos, sin = ang.cos(), ang.sin()

    def rope(x):
        a, b = x[..., :D // 2], x[..., D // 2:]
        return torch.cat([a * cos - b * sin, a * sin + b * cos], -1)

    h = deq(m.embed)[tokens.reshape(-1).long()]
    for sl in sh.layers:
        xn = rms(h)
        q, k, v = (xn @ deq(w).T for w in sl.qkv)
        q = rope(q.view(B, L, -1, D).transpose(1, 2))
        k = rope(k.view(B, L, -1, D).transpose(1, 2))
        v = v.view(B, L, -1, D).transpose(1, 2)
        rep = q.shape[1] // k.shape[1]
        k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1 / math.sqrt(D))
        h = h + o.transpose(1, 2).reshape(B * L, -1) @ deq(sl.o).T
        xn = rms(h)
        g, u = xn @ deq(sl.gate).T, xn @ deq(sl.up).T
        h = h + (F.silu(g) * u) @ deq(sl.down).T
    last = rms(h).view(B, L, -1)[:, -1]
    return last @ deq(sh.lm_head).T


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.fixture(scope="module")
def tp1(cuda):
    return llama_tp.LlamaTP(CFG, 1, [0], llama_tp.LocalComm(), seed=5)


def test_tp1_matches_fp32_restatement(tp1):
    tok = _tokens(2, 192)
    got = tp1(tok)
    torch.cuda.synchronize()
    assert lib.device_status(clear=True) == 0
    ref = _restated(tp1, tok)
    assert got.shape == (2, CFG.vocab)
    assert torch.isfinite(got.float()).all()
    assert _rel(got, ref) < REL_TOL
    assert torch.equal(got.float().argmax(-1), ref.argmax(-1)) or _rel(got, ref) < 1e-2


@pytest.mark.parametrize("tp", [2, 4])
def test_sharded_matches_tp1(tp1, tp):
    tok = _tokens(2, 192)
    ref = tp1(tok)
    sharded = llama_tp.LlamaTP(CFG, tp, range(tp), llama_tp.LocalComm(), seed=5)
    got = sharded(tok)
    torch.cuda.synchronize()
    assert lib.device_status(clear=True) == 0
    assert _rel(got, ref) < 1e-2
    # the shards are slices of the one seeded model
    assert torch.equal(torch.cat([s.lm_head[0] for s in sharded.shards]), tp1.shards[0].lm_head[0])


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_many_rows_forward(tp1, tp):
    """1024 tokens: every projection takes the many-rows form (weights
    dequantised once, tcgen05 GEMM, SwiGLU in the GEMM epilogue) at each
    shard's widths; tp = 1 against the fp32 restatement, tp > 1 against tp = 1."""
    tok = _tokens(2, 512)
    ref = tp1(tok)
    torch.cuda.synchronize()
    if tp == 1:
        assert _rel(ref, _restated(tp1, tok)) < REL_TOL
        return
    sharded = llama_tp.LlamaTP(CFG, tp, range(tp), llama_tp.LocalComm(), seed=5)
    got = sharded(tok)
    torch.cuda.synchronize()
    assert lib.device_status(clear=True) == 0
    assert _rel(got, ref) < 1e-2


def test_forward_is_deterministic(tp1):
    tok = _tokens(1, 128)
    a, b = tp1(tok), tp1(tok)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dims,traditional,H", [(128, False, 6), (64, False, 5), (128, True, 3)])
def test_rope_strided_equals_dense(cuda, dims, traditional, H):
    """mt_rope_strided on the transposed token-major view equals mt_rope on its dense copy, bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(H)
    x = torch.randn(2, 96, H, 128, device="cuda", generator=g).to(torch.bfloat16)  # [B, L, H, D]
    view = x.transpose(1, 2)
    a = lib.rope_bhld(view, dims, traditional=traditional, base=5e5, offset=3)
    b = lib.rope(view.contiguous(), dims, traditional=traditional, base=5e5, offset=3)
    torch.cuda.synchronize()
    assert a.is_contiguous() and torch.equal(a, b)
