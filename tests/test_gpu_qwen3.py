"""The Qwen3 bundle end to end on a small config: every region through the
region contract (try_call -> libmt.so), layer outputs and KV caches against
the oracle's composition of the same regions (oracle/qwen3_ref.py), the
whole request's last-position logits rows, greedy picks and logprob against
the oracle, no fallback taken, and CUDA-graph replay equal to eager
execution."""
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


def test_layer_prefill_then_decode_matches_oracle(model, oracle, strict):
    from oracle import qwen3_ref
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
        ref = qwen3_ref.layer(CFG, qwen3_ref.layer_weights(layer.wrapped), h, kc, vc, off)
        got = n(out)
        tol = 2 ** -6 * np.abs(ref) + 2 ** -7 * np.abs(ref).max()
        assert (np.abs(got - ref) <= tol).all(), np.abs(got - ref).max()
        kv = off + T
        assert np.abs(n(c.k)[:, :kv] - kc[:, :kv]).max() <= 2 ** -6 * np.abs(kc).max()
        assert np.abs(n(c.v)[:, :kv] - vc[:, :kv]).max() <= 2 ** -6 * np.abs(vc).max()
    assert layer.fallbacks == 0


def gpu_request_with_logits(patched, tokens, cache):
    """qwen3.request step by step, keeping each step's last-position logits."""
    cache.reset()
    t0, _ = patched(tokens, cache)
    lg0 = n(patched.last_logits).reshape(-1)
    t1, lp1 = patched(t0, cache)
    lg1 = n(patched.last_logits).reshape(-1)
    return int(t0.item()), lg0, int(t1.item()), float(lp1.item()), lg1


def check_logits(got, ref, tol_frac, label):
    """The whole logits row within tol_frac * max|ref| of the oracle's, and the
    relative L2 error within tol_frac. Returns the absolute tolerance."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    atol = tol_frac * np.abs(ref).max()
    err = np.abs(got - ref)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err.max() <= atol, f"{label}: max |diff| {err.max():.4g} > {atol:.4g} (rel L2 {rel:.3g})"
    assert rel <= tol_frac, f"{label}: relative L2 error {rel:.4g} > {tol_frac}"
    return atol


def check_pick(token, ref_logits, atol, label):
    """The GPU's greedy pick against the oracle's logits: it must be a token
    whose oracle logit is within 2*atol of the oracle's maximum (both sides
    agree on the top to that accuracy), and the argmax itself whenever the
    oracle's top-2 gap exceeds 2*atol. Always asserts something."""
    ref = np.asarray(ref_logits, np.float64)
    top = np.sort(ref)[-2:]
    assert ref[token] >= top[1] - 2 * atol, f"{label}: picked {token}, {top[1] - ref[token]:.4g} below the max"
    if top[1] - top[0] > 2 * atol:
        assert token == int(np.argmax(ref)), f"{label}: clear winner {int(np.argmax(ref))}, picked {token}"


def check_request(oracle, cfg, weights, tokens_np, gpu, tol_frac):
    """A GPU request (gpu_request_with_logits) against the oracle composition,
    the oracle's decode step fed the GPU's first pick."""
    from oracle import qwen3_ref
    t0, lg0, t1, lp1, lg1 = gpu
    ref = qwen3_ref.request(cfg, weights, tokens_np, force_token0=t0)
    a0 = check_logits(lg0, ref.prefill_logits, tol_frac, "prefill logits")
    check_pick(t0, ref.prefill_logits, a0, "prefill pick")
    a1 = check_logits(lg1, ref.decode_logits, tol_frac, "decode logits")
    check_pick(t1, ref.decode_logits, a1, "decode pick")
    # logprob of the GPU's pick under the oracle's logits (lse in fp32, the difference rounded to bf16)
    r = ref.decode_logits.astype(np.float64)
    lse = np.log(np.exp(r - r.max()).sum()) + r.max()
    lp_ref = float(oracle.round_to(np.array([r[t1] - lse], np.float32), "bfloat16")[0])
    assert abs(lp1 - lp_ref) <= 2 * a1 + 2 ** -7 * abs(lp_ref), (lp1, lp_ref)
    return ref


REQUEST_TOL = 2 ** -5  # bf16 activations through 2 layers, reordered fp32 sums in every region


def test_request_matches_oracle_logits(model, oracle, strict):
    from oracle import qwen3_ref
    patched = apply(model, BUNDLE)
    cache = qwen3.KVCache(CFG, device="cuda")
    tokens = torch.randint(0, CFG.vocab, (32,), dtype=torch.int32, generator=torch.Generator().manual_seed(9)).cuda()
    gpu = gpu_request_with_logits(patched, tokens, cache)
    check_request(oracle, CFG, qwen3_ref.model_weights(model), tokens.cpu().numpy(), gpu, REQUEST_TOL)
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
