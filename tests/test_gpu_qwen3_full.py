"""The full Qwen3-4B-4bit config the benchmark times (36 layers, hidden 2560,
32/8 heads, FFN 9728, vocab 151936, 4-bit g64), with the benchmark's seeds:
the bundle's layer 0 at prefill (128 tokens) and decode (1 token at offset
128), and the whole request's logits rows, picks and logprob, against the
oracle composition of the same regions (oracle/qwen3_ref.py) on the same
weights copied to the host. The oracle runs the whole 36-layer request on
the host cores (about 20 s)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from metal_autotune_b200 import workload
from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.targets import qwen3

from test_gpu_qwen3 import check_request, gpu_request_with_logits, n

pytestmark = pytest.mark.gpu

BUNDLE = Path(__file__).resolve().parents[1] / "metal_autotune_b200" / "bundles" / "qwen3_4b"
CFG = qwen3.QWEN3_4B
SEED = 0          # bench.py Request(cfg, seed=0): model and prompt
LAYER_TOL = 2 ** -6
REQUEST_TOL = 2 ** -4  # 36 layers of bf16 activations, reordered fp32 sums in every region


@pytest.fixture(scope="module")
def full(cuda):
    model = qwen3.build(CFG, seed=SEED, device="cuda")
    from oracle import qwen3_ref
    weights = qwen3_ref.model_weights(model)
    return model, weights


@pytest.fixture()
def strict(monkeypatch):
    monkeypatch.setenv("MT_STRICT_REGIONS", "1")


def test_full_config_layer0_prefill_and_decode(full, oracle, strict):
    from oracle import qwen3_ref
    model, weights = full
    patched = apply(model, BUNDLE)
    layer = patched.wrapped.layers[0]
    cache = qwen3.KVCache(CFG, device="cuda")
    c = cache.layers[0]
    kc, vc = qwen3_ref.empty_cache(CFG)[0]
    tokens = workload.seeded_tokens((128,), 0, CFG.vocab, seed=SEED)
    E = weights.embed
    h = oracle.quantized_embedding(tokens.cpu().numpy(), E.wq, E.scales, E.biases, CFG.group, CFG.bits)
    for T, off, x in ((128, 0, h), (1, 128, h[-1:])):
        c.offset = off
        got = n(layer(torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda(), c))
        ref = qwen3_ref.layer(CFG, weights.layers[0], x, kc, vc, off)
        tol = LAYER_TOL * np.abs(ref) + 2 ** -7 * np.abs(ref).max()
        bad = np.abs(got - ref) > tol
        assert not bad.any(), f"T={T}: {bad.sum()} outside, worst {np.abs(got - ref).max():.4g}"
        kv = off + T
        assert np.abs(n(c.k)[:, :kv] - kc[:, :kv]).max() <= LAYER_TOL * np.abs(kc).max()
        assert np.abs(n(c.v)[:, :kv] - vc[:, :kv]).max() <= LAYER_TOL * np.abs(vc).max()
    assert layer.fallbacks == 0


def test_full_config_request_logits(full, oracle, strict):
    model, weights = full
    patched = apply(model, BUNDLE)
    cache = qwen3.KVCache(CFG, device="cuda")
    tokens = workload.seeded_tokens((128,), 0, CFG.vocab, seed=SEED)
    gpu = gpu_request_with_logits(patched, tokens, cache)
    check_request(oracle, CFG, weights, tokens.cpu().numpy(), gpu, REQUEST_TOL)
    assert patched.fallbacks == 0 and all(l.fallbacks == 0 for l in patched.wrapped.layers)
