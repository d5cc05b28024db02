"""Host-side checks of the whole-model targets and their oracle compositions:
the torch module trees (the original op sequences a region wrapper falls back
to) built on the CPU against the oracle's composition of the same regions,
at small configs. Both are restatements with different summation orders, so
they agree within the rounding of the element type."""
from __future__ import annotations

import numpy as np
import pytest
import torch


def _close(got, ref, ulp, k=3, kmax=2):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    tol = k * ulp * np.abs(ref) + kmax * ulp * np.abs(ref).max()
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside; worst {np.abs(got - ref).max():.4g}"


def test_whisper_tiny_original_ops_match_oracle():
    from metal_autotune_b200.targets import whisper
    from oracle import whisper_ref
    cfg = whisper.TINY
    enc = whisper.build(cfg, seed=1, device="cpu")
    mel = torch.randn(2, cfg.frames, cfg.n_mels, generator=torch.Generator().manual_seed(2)).to(torch.float16)
    with torch.no_grad():
        got = enc(mel).float().numpy()
    ref = whisper_ref.encoder(cfg, whisper_ref.encoder_weights(enc), mel.float().numpy())
    # two blocks of fp16 activations, reordered fp32 sums in every linear
    _close(got, ref, 2.0 ** -10, k=8, kmax=4)


def test_whisper_sinusoids_are_the_published_table():
    from metal_autotune_b200.targets import whisper
    t = whisper.sinusoids(1500, 1280)
    assert t.shape == (1500, 1280)
    # position 0: sin 0 = 0 and cos 0 = 1; the last frequency is 1e-4 rad per position
    assert torch.all(t[0, :640] == 0) and torch.all(t[0, 640:] == 1)
    assert abs(float(t[1499, 639]) - np.sin(1499 * 1e-4)) < 1e-6


def test_whisper_flops_count():
    from metal_autotune_b200.targets import whisper
    f = whisper.encoder_flops(whisper.WHISPER_TURBO, 8)
    assert 17e12 < f < 19e12  # ~15.1 TFLOP of projections/MLP/conv + ~2.9 of attention


def test_mamba_tiny_original_ops_match_oracle():
    from metal_autotune_b200.targets import mamba
    from oracle import mamba_ref
    cfg = mamba.TINY
    model = mamba.build(cfg, seed=1, device="cpu")
    tok = torch.randint(0, cfg.vocab, (24,), generator=torch.Generator().manual_seed(3), dtype=torch.int32)
    with torch.no_grad():
        t, logits = model(tok)
    ref, rt = mamba_ref.prefill(cfg, mamba_ref.model_weights(model), tok.numpy())
    _close(logits.float().numpy().reshape(-1), ref, 2.0 ** -10, k=8, kmax=4)


def test_mamba_flops_count():
    from metal_autotune_b200.targets import mamba
    f = mamba.prefill_flops(mamba.MAMBA_370M, 512)
    assert 0.3e12 < f < 0.4e12
