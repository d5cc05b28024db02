"""Graph-backend bundles on the GPU: the traced, rewritten graph of each
target runs every region through libmt.so, with no fallback (strict), and
agrees with the replay bundle of the same target and with the oracle.

The tiny MLP's graph runs the same two kernels on the same inputs as its
replay bundle, so the outputs are bit-identical. The Whisper graph computes
q, k and v as three linears where the replay bundle runs one GEMM over the
stacked weights; both are checked against the oracle composition with the
replay test's tolerance (fp16 ulp 2^-10: 8 ulp relative plus 2 ulp of the
largest magnitude per block)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib
from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.targets import tiny_mlp, whisper

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


def test_tiny_mlp_graph_equals_replay_bundle(cuda, strict):
    model, x = tiny_mlp.build()
    replay = apply(model, BUNDLES / "tiny_mlp")
    want = replay(x)
    graph = apply(tiny_mlp.build()[0], BUNDLES / "tiny_mlp_graph")
    graph(x)  # first call traces and rewrites
    before = lib.CALLS[0]
    got = graph(x)
    torch.cuda.synchronize()
    assert lib.CALLS[0] - before == 2  # the two regions, nothing else through libmt
    assert torch.equal(got, want)


def test_whisper_tiny_graph_matches_oracle_and_replay(cuda, oracle, strict):
    from oracle import whisper_ref
    cfg = whisper.TINY
    enc = whisper.build(cfg, seed=1)
    W = whisper_ref.encoder_weights(enc)
    mel = torch.randn(2, cfg.frames, cfg.n_mels, generator=torch.Generator().manual_seed(2)).to(torch.float16)
    graph = apply(enc, BUNDLES / "whisper_tiny_graph")
    got = graph(mel.cuda())
    before = lib.CALLS[0]
    again = graph(mel.cuda())
    torch.cuda.synchronize()
    n = cfg.n_layer
    assert lib.CALLS[0] - before == 3 + 9 * n + 1  # stem (3), per block 9 regions, ln_post
    assert torch.equal(got, again)
    ref = whisper_ref.encoder(cfg, W, mel.float().numpy())
    close(got.float().cpu().numpy(), ref, k=8, kmax=2 * n)
    replay = apply(whisper.build(cfg, seed=1), BUNDLES / "whisper_tiny")(mel.cuda())
    close(got.float().cpu().numpy(), replay.float().cpu().numpy(), k=8, kmax=2 * n)


def test_whisper_tiny_graph_captures_in_a_cuda_graph(cuda, strict):
    cfg = whisper.TINY
    graph = apply(whisper.build(cfg, seed=3), BUNDLES / "whisper_tiny_graph")
    mel = torch.randn(2, cfg.frames, cfg.n_mels, device="cuda").to(torch.float16)
    eager = graph(mel).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph(mel)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = graph(mel)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_whisper_turbo_graph_one_clip_matches_replay(cuda, strict):
    """whisper-large-v3-turbo (32 blocks, 1280 state, 20 heads), one clip:
    the graph backend against the replay bundle on the same weights."""
    cfg = whisper.WHISPER_TURBO
    enc = whisper.build(cfg, seed=0)
    mel = torch.randn(1, cfg.frames, cfg.n_mels, generator=torch.Generator().manual_seed(4)).to(torch.float16).cuda()
    graph = apply(enc, BUNDLES / "whisper_turbo_graph")
    got = graph(mel).float().cpu().numpy()
    hits = {e["kernel_id"]: e["hits"] for e in graph._graph_evidence[-1]}
    assert hits["layer_norm"] == 2 * cfg.n_layer + 1 and hits["attention"] == cfg.n_layer
    want = apply(whisper.build(cfg, seed=0), BUNDLES / "whisper_turbo")(mel).float().cpu().numpy()
    close(got, want, k=8, kmax=2 * cfg.n_layer)
