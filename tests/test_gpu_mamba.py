"""The Mamba bundle end to end: every region through the region contract
(try_call -> libmt.so: tcgen05 GEMMs for the projections, the depthwise
causal conv, the chunked selective scan, RMSNorm, the embedding gather, the
lm_head and the greedy pick), against the oracle's composition of the same
regions (oracle/mamba_ref.py) with no fallback taken, CUDA-graph replay equal
to eager execution, and one layer at the full Mamba-370m width over 512
tokens.

Tolerance: fp16 activations (ulp 2^-10), reordered fp32 sums, the scan's
exponentials from the device library: 8 ulp relative plus 4 ulp of the
largest magnitude per layer of depth."""
from pathlib import Path

import numpy as np
import pytest
import torch

from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.targets import mamba

pytestmark = pytest.mark.gpu

BUNDLES = Path(__file__).resolve().parents[1] / "metal_autotune_b200" / "bundles"
ULP = 2.0 ** -10


def close(got, ref, k=8, kmax=4):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    tol = k * ULP * np.abs(ref) + kmax * ULP * np.abs(ref).max()
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside; worst {np.abs(got - ref).max():.4g}"


@pytest.fixture()
def strict(monkeypatch):
    monkeypatch.setenv("MT_STRICT_REGIONS", "1")


def test_tiny_prefill_matches_oracle(cuda, oracle, strict):
    from oracle import mamba_ref
    cfg = mamba.TINY
    model = mamba.build(cfg, seed=1)
    W = mamba_ref.model_weights(model)
    patched = apply(model, BUNDLES / "mamba_tiny")
    tok = torch.randint(0, cfg.vocab, (96,), generator=torch.Generator().manual_seed(3), dtype=torch.int32)
    t, logits = patched(tok.cuda())
    ref, rt = mamba_ref.prefill(cfg, W, tok.numpy())
    close(logits.float().cpu().numpy().reshape(-1), ref, k=8, kmax=4 * cfg.n_layer)
    got_t = int(t.item())
    gap = np.sort(ref)[-1] - ref[got_t]
    assert gap <= 8 * cfg.n_layer * ULP * np.abs(ref).max()  # the pick is a top logit of the oracle's row
    assert patched.fallbacks == 0 and all(l.fallbacks == 0 for l in patched.wrapped.layers)


def test_tiny_graph_replay_equals_eager(cuda, strict):
    cfg = mamba.TINY
    patched = apply(mamba.build(cfg, seed=2), BUNDLES / "mamba_tiny")
    tok = torch.randint(0, cfg.vocab, (64,), dtype=torch.int32, device="cuda")
    eager = [x.clone() for x in patched(tok)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        patched(tok)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = patched(tok)
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, out):
        assert torch.equal(a, b)


def test_full_width_layer(cuda, oracle, strict):
    """Mamba-370m widths (d_model 1024, d_inner 2048, d_state 16, dt_rank 64),
    layer 0 over 512 tokens through the bundle's regions."""
    from oracle import mamba_ref
    cfg = mamba.MAMBA_370M
    model = mamba.build(cfg, seed=0)
    patched = apply(model, BUNDLES / "mamba_370m")
    W = mamba_ref.model_weights(model, n_layers=1)
    x = (torch.randn(512, cfg.d_model, generator=torch.Generator().manual_seed(5)) * 0.5).to(torch.float16)
    got = patched.wrapped.layers[0](x.cuda()).float().cpu().numpy()
    ref = mamba_ref.layer(cfg, W.layers[0], x.float().numpy())
    close(got, ref, k=8, kmax=4)
    assert patched.wrapped.layers[0].fallbacks == 0
