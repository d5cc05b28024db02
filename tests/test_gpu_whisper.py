"""The Whisper encoder bundle end to end: every region through the region
contract (try_call -> libmt.so: tcgen05 implicit-GEMM convs and linears,
tcgen05 flash attention, LayerNorm, positional add), against the oracle's
composition of the same regions (oracle/whisper_ref.py), with no fallback
taken; CUDA-graph replay equal to eager execution; and, at the full
whisper-large-v3-turbo width, the stem and the first block of one clip.

Tolerance: fp16 activations (ulp 2^-10) with reordered fp32 sums in every
linear and in the attention, P rounded to fp16 before P.V: 8 ulp relative
plus 4 ulp of the tensor's largest magnitude per block of depth."""
from pathlib import Path

import numpy as np
import pytest
import torch

from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.targets import whisper

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


def test_tiny_encoder_matches_oracle(cuda, oracle, strict):
    from oracle import whisper_ref
    cfg = whisper.TINY
    enc = whisper.build(cfg, seed=1)
    W = whisper_ref.encoder_weights(enc)
    patched = apply(enc, BUNDLES / "whisper_tiny")
    mel = torch.randn(2, cfg.frames, cfg.n_mels, generator=torch.Generator().manual_seed(2)).to(torch.float16)
    got = patched(mel.cuda()).float().cpu().numpy()
    ref = whisper_ref.encoder(cfg, W, mel.float().numpy())
    close(got, ref, k=8, kmax=2 * cfg.n_layer)
    assert patched.fallbacks == 0 and all(b.fallbacks == 0 for b in patched.wrapped.blocks)


def test_tiny_encoder_graph_replay_equals_eager(cuda, strict):
    cfg = whisper.TINY
    patched = apply(whisper.build(cfg, seed=3), BUNDLES / "whisper_tiny")
    mel = torch.randn(2, cfg.frames, cfg.n_mels, device="cuda").to(torch.float16)
    eager = patched(mel).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        patched(mel)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = patched(mel)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_full_width_stem_and_first_block(cuda, oracle, strict):
    """whisper-large-v3-turbo widths (1280 state, 20 heads, 1500 positions),
    one clip, the stem and block 0 through the bundle's regions."""
    from oracle import whisper_ref
    cfg = whisper.WHISPER_TURBO
    enc = whisper.build(cfg, seed=0)
    patched = apply(enc, BUNDLES / "whisper_turbo")
    mel = torch.randn(1, cfg.frames, cfg.n_mels, generator=torch.Generator().manual_seed(4)).to(torch.float16)
    W = whisper_ref.encoder_weights(enc, n_blocks=1)
    E = patched.wrapped
    x = mel.cuda()
    r = [patched._call(k, a) for k, a in [("conv1_gelu", [x, E.conv1.weight, E.conv1.bias])]][0]
    r = patched._call("conv2_gelu", [r[0], E.conv2.weight, E.conv2.bias])
    r = patched._call("pos_add", [r[0], E.positional_embedding])
    stem_ref = whisper_ref.stem(cfg, W, mel.float().numpy())
    close(r[0].float().cpu().numpy(), stem_ref, k=8, kmax=2)
    blk = E.blocks[0](r[0]).float().cpu().numpy()
    close(blk, whisper_ref.block(cfg, W.blocks[0], stem_ref), k=8, kmax=4)
    assert E.blocks[0].fallbacks == 0
