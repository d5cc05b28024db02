"""Region pricing on the GPU: the region clock (recorded calls replayed on
real tensors, L2 flushed before every sample, CUDA events) and the step
clock, for the tiny Whisper encoder's non-overlapping candidate wave."""
import pytest
import torch

from metal_autotune_b200 import regions as R
from metal_autotune_b200.targets import whisper

pytestmark = pytest.mark.gpu


def test_price_and_rank_the_whisper_wave(cuda):
    cfg = whisper.TINY
    model = whisper.build(cfg, seed=0)
    x = torch.randn(2, cfg.frames, cfg.n_mels, device="cuda").half()
    t, regions = R.discover(model, (x,), "w")
    pk = R.roofline.peaks()
    est = R.price.estimate(t, regions, pk)
    wave, _ = R.rank.select_frontier(regions, lambda r: est[r.fingerprint][1])
    step_ms = R.price.price(t, wave, model, (x,), pk)
    assert step_ms > 0
    for r in wave:
        assert r.t_rep_ms["w"] > 0 and r.roofline is not None
        assert r.p["w"] == pytest.approx(r.t_rep_ms["w"] * r.copies / step_ms)
        assert r.roofline.s_max == pytest.approx(r.t_rep_ms["w"] / r.roofline.t_roofline_ms)
    # the wave does not overlap, so its copies' shares add up to about one step
    # (each region replayed alone pays its own launches and cold L2)
    total = sum(r.combined_p for r in wave)
    assert 0.3 < total < 3.0, total
    ranked = R.rank.rank(R.rank.apply_floor(wave))
    assert ranked
    scores = [r.combined_removable_p * R.rank.length_weight(r) for r in ranked]
    assert scores == sorted(scores, reverse=True)


def test_replayed_copy_computes_what_the_model_computes(cuda):
    cfg = whisper.TINY
    model = whisper.build(cfg, seed=0)
    x = torch.randn(2, cfg.frames, cfg.n_mels, device="cuda").half()
    t = R.trace.record(model, (x,), "w")
    weights = dict(model.named_buffers())
    weights.update(dict(model.named_parameters()))
    bound = {aid: weights[p] for aid, p in t.weights.items()}
    bound[t.inputs[0]] = x
    env = R.trace.replay(t, 0, len(t.nodes) - 1, bound)
    assert torch.equal(env[t.step_outputs[0]], model(x))
