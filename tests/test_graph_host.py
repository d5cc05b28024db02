"""Graph-backend bundles on the host: tracing, rule counts, fallbacks and
structure proofs run on the CPU (the rewritten graphs' region calls need a
GPU; tests/test_gpu_graph.py runs them)."""
import copy
import json

import pytest
import torch

from metal_autotune_b200.autotuner_runtime import graph as graph_rt
from metal_autotune_b200.autotuner_runtime import graph_native as G
from metal_autotune_b200.autotuner_runtime.apply import apply
from metal_autotune_b200.bundles import HERE
from metal_autotune_b200.targets import tiny_mlp, whisper


def _whisper_tiny():
    model = whisper.build(whisper.TINY, seed=0, device="cpu")
    return model, apply(model, HERE / "whisper_tiny_graph")


def test_whisper_rules_replace_every_region_with_the_recorded_counts():
    _, g = _whisper_tiny()
    x = torch.randn(2, whisper.TINY.frames, whisper.TINY.n_mels).half()
    assert g.regions_left((x,)) == []
    n = whisper.TINY.n_layer
    hits = {e["kernel_id"]: e["hits"] for e in g._graph_evidence[-1]}
    assert hits == {"conv1_gelu": 1, "conv2_gelu": 1, "pos_add": 1, "fc1_gelu": n, "fc2_residual": n,
                    "out_proj_residual": n, "attention": n, "linear_bias": 2 * n, "linear_nobias": n,
                    "layer_norm": 2 * n + 1}
    gm = g.build_graph((x,), g.variant_for((x,))["rules"])
    regions = [m for _, m in gm.named_children() if isinstance(m, graph_rt.RegionCall)]
    assert len(regions) == sum(hits.values())


def test_tiny_mlp_rules_leave_no_op_outside_a_region():
    model, x = tiny_mlp.build(device="cpu")
    g = apply(model, HERE / "tiny_mlp_graph")
    assert g.regions_left((x,)) == []
    assert [e["hits"] for e in g._graph_evidence[-1]] == [1, 1]


def test_unrecorded_signature_runs_the_original(monkeypatch):
    monkeypatch.delenv("MT_STRICT_REGIONS", raising=False)
    model, g = _whisper_tiny()
    x = torch.randn(1, whisper.TINY.frames, whisper.TINY.n_mels).half()  # batch 1 is not recorded
    out = g(x)
    assert torch.equal(out, model(x))
    assert "no recorded variant" in g._graph_fallbacks[-1]
    monkeypatch.setenv("MT_STRICT_REGIONS", "1")
    g2 = apply(whisper.build(whisper.TINY, seed=0, device="cpu"), HERE / "whisper_tiny_graph")
    with pytest.raises(graph_rt.GraphBindingError):
        g2(x)


def test_a_rule_count_that_no_longer_holds_sends_the_call_to_the_original(monkeypatch):
    monkeypatch.delenv("MT_STRICT_REGIONS", raising=False)
    model, x = tiny_mlp.build(device="cpu")
    g = apply(model, HERE / "tiny_mlp_graph")
    variants = copy.deepcopy(list(type(g).GRAPH_VARIANTS))
    variants[0]["rules"][1]["count"] = 2  # the graph holds one second linear
    object.__setattr__(g, "GRAPH_VARIANTS", tuple(variants))
    out = g(x)  # CPU: the original module's forward
    assert torch.equal(out, model(x))
    assert "replaced 1 graph cuts, expected 2" in g._graph_fallbacks[-1]


def test_two_builds_of_the_same_target_trace_the_same_computation():
    a, b = whisper.build(whisper.TINY, seed=0, device="cpu"), whisper.build(whisper.TINY, seed=1, device="cpu")
    x = torch.randn(2, whisper.TINY.frames, whisper.TINY.n_mels).half()
    names = [n for n, _, _ in graph_rt._weights(a)]
    ga, gb = graph_rt.trace(a, (x,), names), graph_rt.trace(b, (x,), names)
    assert G.same_structure(ga, gb)[0]
    assert G.same_computation(ga, gb)[0]
    # another head count is another computation
    c = whisper.build(whisper.WhisperConfig(n_mels=128, n_ctx=200, n_state=256, n_head=8, n_layer=2), seed=0,
                      device="cpu")
    gc = graph_rt.trace(c, (x,), names)
    same, why = G.same_structure(ga, gc)
    assert not same and why


def test_graph_variants_file_matches_the_generator():
    from metal_autotune_b200 import bundles
    recorded = json.loads((HERE / "whisper_turbo_graph" / "patch" / "graph_variants.json").read_text())
    assert recorded == json.loads(json.dumps(bundles.whisper_graph_variants(whisper.WHISPER_TURBO, (1, 8))))
    batches = [v["args"][0][0][0] for v in recorded["G_whisper_encoder"]]
    assert batches == [1, 8]
