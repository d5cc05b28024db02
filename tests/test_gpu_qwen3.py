"""The Qwen3 bundle end to end on a small config: every region through the
region contract (try_call -> libmt.so), layer outputs and KV caches against
the oracle's composition of the same regions, the whole request's picked
tokens against the oracle, no fallback taken, and CUDA-graph replay equal to
eager execution."""
import math
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.targets import qwen3

pytestmark = pytest.mark.gpu

BUNDLE = Path(__file__).resolve().parents[1] / "metal_autotune_b200" / "bundles" / "qwen3_tiny"
CFG = qwen3.TINY


def n(x):
    return x.float().cpu().numpy()


def u32(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.fixture()
def strict(monkeypatch):
    monkeypatch.setenv("MT_STRICT_REGIONS", "1")


@pytest.fixture(scope="module")
def model(cuda):
    torch.manual_seed(0)
    return qwen3.build(CFG, seed=3, device="cuda")


def oracle_layer(R, L, h, kc, vc, offset):
    """The layer's regions composed from oracle restatements (numpy)."""
    a, m = L.self_attn, L.mlp
    T = h.shape[0]
    qm = lambda x, p: R.quantized_matmul(x, u32(p.weight), n(p.scales), n(p.biases), CFG.group, CFG.bits)
    xn = R.rms_norm(h, n(L.input_layernorm.weight), CFG.eps)
    q, k, v = qm(xn, a.q_proj), qm(xn, a.k_proj), qm(xn, a.v_proj)
    qh, kc, vc = R.qk_norm_rope_cache(q, k, v, n(a.q_norm.weight), n(a.k_norm.weight), CFG.eps, kc, vc,
                                      CFG.heads, CFG.kv_heads, offset, CFG.rope_theta)
    kv = offset + T
    o = R.sdpa(qh[None], kc[None, :, :kv], vc[None, :, :kv], 1 / math.sqrt(CFG.head_dim), True, offset)
    o = o[0].transpose(1, 0, 2).reshape(T, -1)
    h2 = R.add(qm(o, a.o_proj), h)
    xn2 = R.rms_norm(h2, n(L.post_attention_layernorm.weight), CFG.eps)
    act = R.swiglu(qm(xn2, m.gate_proj), qm(xn2, m.up_proj))
    return R.add(qm(act, m.down_proj), h2)


def test_layer_prefill_then_decode_matches_oracle(model, oracle, strict):
    patched = apply(model, BUNDLE)
    layer = patched.wrapped.layers[0]
    cache = qwen3.KVCache(CFG, device="cuda")
    c = cache.layers[0]
    rng = np.random.default_rng(5)
    kc = np.zeros((CFG.kv_heads, CFG.max_len, CFG.head_dim), np.float32)
    vc = np.zeros_like(kc)
    for T, off in ((32, 0), (1, 32)):
        h = oracle.round_to(rng.standard_normal((T, CFG.hidden)).astype(np.float32), "bfloat16")
        c.offset = off
        out = layer(torch.from_numpy(h).to(torch.bfloat16).cuda(), c)
        ref = oracle_layer(oracle, layer.wrapped, h, kc, vc, off)
        got = n(out)
        tol = 2 ** -6 * np.abs(ref) + 2 ** -7 * np.abs(ref).max()
        assert (np.abs(got - ref) <= tol).all(), np.abs(got - ref).max()
        kv = off + T
        assert np.abs(n(c.k)[:, :kv] - kc[:, :kv]).max() <= 2 ** -6 * np.abs(kc).max()
        assert np.abs(n(c.v)[:, :kv] - vc[:, :kv]).max() <= 2 ** -6 * np.abs(vc).max()
    assert layer.fallbacks == 0


def test_request_matches_oracle_tokens(model, oracle, strict):
    patched = apply(model, BUNDLE)
    cache = qwen3.KVCache(CFG, device="cuda")
    tokens = torch.randint(0, CFG.vocab, (32,), dtype=torch.int32, generator=torch.Generator().manual_seed(9)).cuda()
    t0, t1, lp1 = qwen3.request(patched, tokens, cache)
    # oracle request
    E = model.embed_tokens
    ew, es, eb = u32(E.weight), n(E.scales), n(E.biases)
    kcs = [np.zeros((CFG.kv_heads, CFG.max_len, CFG.head_dim), np.float32) for _ in range(CFG.layers)]
    vcs = [np.zeros_like(k) for k in kcs]

    def step(tok, off):
        h = oracle.quantized_embedding(tok, ew, es, eb, CFG.group, CFG.bits)
        for i, L in enumerate(model.layers):
            h = oracle_layer(oracle, L, h, kcs[i], vcs[i], off)
        last = oracle.rms_norm(h[-1:], n(model.norm.weight), CFG.eps)
        logits = oracle.quantized_matmul(last, ew, es, eb, CFG.group, CFG.bits)
        return logits.reshape(-1)

    lg0 = step(tokens.cpu().numpy(), 0)
    r0 = int(np.argmax(lg0))
    top = np.sort(lg0)[-2:]
    if top[1] - top[0] > 0.05 * abs(top[1]):  # a clear winner must agree
        assert int(t0.item()) == r0
    lg1 = step(np.array([int(t0.item())], np.int32), 32)
    tok1, lp, _ = oracle.logits_pick(lg1)
    top = np.sort(lg1)[-2:]
    if top[1] - top[0] > 0.05 * abs(top[1]):
        assert int(t1.item()) == tok1
        assert abs(float(lp1.item()) - lp) <= 0.05 * abs(lp) + 0.05
    assert patched.fallbacks == 0 and all(l.fallbacks == 0 for l in patched.wrapped.layers)


def test_unpatched_model_agrees_within_tolerance(model, strict):
    """The region kernels against the original torch op sequence (the thing
    they replace): first-layer outputs agree to bf16 rounding."""
    patched = apply(model, BUNDLE)
    h = torch.randn(16, CFG.hidden, device="cuda").to(torch.bfloat16)
    c1 = qwen3.KVCache(CFG, device="cuda").layers[0]
    c2 = qwen3.KVCache(CFG, device="cuda").layers[0]
    a = patched.wrapped.layers[0](h, c1)
    b = patched.wrapped.layers[0].wrapped(h, c2)
    err = (a.float() - b.float()).abs().max().item()
    assert err <= 0.05 * b.float().abs().max().item()


def test_graph_replay_equals_eager(model, strict):
    patched = apply(model, BUNDLE)
    cache = qwen3.KVCache(CFG, device="cuda")
    tokens = torch.randint(0, CFG.vocab, (32,), dtype=torch.int32, device="cuda")
    eager = [x.clone() for x in qwen3.request(patched, tokens, cache)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        qwen3.request(patched, tokens, cache)  # warm: workspaces and launch caches exist before capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = qwen3.request(patched, tokens, cache)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, out):
        assert torch.equal(a, b)
