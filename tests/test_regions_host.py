"""Region discovery on the host (recording on fake tensors, stretches,
copy grouping, roofline arithmetic, ranking): no GPU involved."""
import torch

from metal_autotune_b200 import regions as R
from metal_autotune_b200.autotuner_runtime.graph import sequence_of
from metal_autotune_b200.bundles import whisper_graph_variants
from metal_autotune_b200.regions import build as B
from metal_autotune_b200.targets import tiny_mlp, whisper


def _whisper():
    cfg = whisper.TINY
    model = whisper.build(cfg, seed=0, device="cpu")
    x = torch.randn(2, cfg.frames, cfg.n_mels, generator=torch.Generator().manual_seed(0)).half()
    return cfg, model, x


def test_trace_records_aten_calls_with_scopes_and_weights():
    model, x = tiny_mlp.build(device="cpu")
    t = R.trace.record(model, (x,), "tiny_mlp")
    ops = [B.base(n.op) for n in t.nodes]
    assert ops.count("mm") == 2 and "erf" in ops
    assert set(t.weights.values()) == {"l1.weight", "l1.bias", "l2.weight", "l2.bias"}
    mm = [n for n in t.nodes if B.base(n.op) == "mm"]
    assert mm[0].module_address == "l1" and mm[1].module_address == "l2"
    assert len(t.step_outputs) == 1 and t.specs[t.step_outputs[0]] == ((32, 256), "float32")


def test_replaying_the_whole_trace_reproduces_the_forward():
    cfg, model, x = _whisper()
    t = R.trace.record(model, (x,), "w")
    weights = dict(model.named_buffers())
    weights.update(dict(model.named_parameters()))
    bound = {aid: weights[path] for aid, path in t.weights.items()}
    bound[t.inputs[0]] = x
    env = R.trace.replay(t, 0, len(t.nodes) - 1, bound)
    assert torch.equal(env[t.step_outputs[0]], model(x))


def test_no_region_holds_a_product_fed_by_another_product():
    cfg, model, x = _whisper()
    t, regions = R.discover(model, (x,), "w")
    for r in regions:
        for s in r.members:
            nodes = t.nodes[s.start_seq:s.end_seq + 1]
            down = set()
            for n in nodes:
                reads = any(a in down for a in n.in_arrays)
                assert not (B.is_matmul_like(n) and reads), r.ops
                if B.is_matmul_like(n) or reads:
                    down.update(n.out_arrays)


def test_discovery_finds_the_graph_bundle_regions_with_their_counts():
    """Each graph rule's pattern is a discovered region with as many copies
    as the rule replaces; the biased [S, S] linear also has the out
    projection's copy (the out_proj_residual rule consumes it first), and
    the positional add starts on no anchor (it follows GELU in the same
    scope and reads an activation first)."""
    cfg, model, x = _whisper()
    t, regions = R.discover(model, (x,), "w")
    by = {r.fingerprint: r for r in regions}
    weights = {"conv1_gelu": (1, 2), "conv2_gelu": (1, 2), "fc1_gelu": (1, 2), "fc2_residual": (1, 2),
               "out_proj_residual": (1, 2), "attention": (), "linear_bias": (1, 2), "linear_nobias": (1,),
               "layer_norm": (1, 2)}
    extra = {"linear_bias": cfg.n_layer}
    for rule in whisper_graph_variants(cfg, (2,))["G_whisper_encoder"][0]["rules"]:
        kid = rule["kernel_id"]
        if kid == "pos_add":
            continue
        ins = [torch.randn(s).to(getattr(torch, d)) for s, d in rule["input_specs"]]
        fp = R.pattern_fingerprint(sequence_of(rule), ins, weights[kid])
        assert fp in by, kid
        assert by[fp].copies == rule["count"] + extra.get(kid, 0), kid


def test_copies_are_grouped_across_layers_and_sizes():
    cfg, model, x = _whisper()
    t, regions = R.discover(model, (x,), "w")
    fc1 = R.pattern_fingerprint(whisper.linear_gelu, [torch.randn(2, 200, 256).half(),
                                                      torch.randn(1024, 256).half(), torch.randn(1024).half()], (1, 2))
    r = next(r for r in regions if r.fingerprint == fc1)
    # fc1 runs in blocks.i.mlp1 and GELU in the block's own forward: the copy's scope is the block
    assert [m.scope_stack[-1] for m in r.members] == ["blocks.0", "blocks.1"]
    # the same sequence at another activation size is the same region; another weight shape is not
    same = R.pattern_fingerprint(whisper.linear_gelu, [torch.randn(1, 50, 256).half(),
                                                       torch.randn(1024, 256).half(), torch.randn(1024).half()], (1, 2))
    other = R.pattern_fingerprint(whisper.linear_gelu, [torch.randn(2, 200, 256).half(),
                                                        torch.randn(512, 256).half(), torch.randn(512).half()], (1, 2))
    assert same == fc1 and other != fc1


def test_roofline_flops_of_the_products_are_the_encoder_flops():
    cfg, model, x = _whisper()
    t = R.trace.record(model, (x,), "w")
    products = sum(R.roofline.node_flops(n) for n in t.nodes
                   if B.is_matmul_like(n))
    assert products == whisper.encoder_flops(cfg, 2)
    pk = R.roofline.Peaks(6445.0, {"float16": 1684.3, "bfloat16": 1684.3, "float32": 74.4}, 2.0, "test")
    floor = R.roofline.step_floor(t, pk, 1.0)
    assert floor["floor_ms"] == max(floor["t_mem_ms"], floor["t_compute_ms"]) and 0 < floor["room"] < 1


def test_rank_orders_by_removable_share_and_frontier_does_not_overlap():
    cfg, model, x = _whisper()
    t, regions = R.discover(model, (x,), "w")
    pk = R.roofline.peaks()
    est = R.price.estimate(t, regions, pk)
    ready, deferred = R.rank.select_frontier(regions, lambda r: est[r.fingerprint][1])
    for i, a in enumerate(ready):
        for b in ready[i + 1:]:
            assert not R.rank._overlap(a, b)
    assert set(deferred) | {r.fingerprint for r in ready} == {r.fingerprint for r in regions}
    # ranking of priced regions: removable share p(1 - 1/s_max), weighted by length
    for i, r in enumerate(regions[:6]):
        r.p = {"w": 0.05 * (i + 1)}
        r.roofline = R.roofline.Roofline(0, 0, 0, 1.0, "compute", 2.0)
    ranked = R.rank.rank(R.rank.apply_floor(regions[:6]))
    scores = [r.combined_removable_p * R.rank.length_weight(r) for r in ranked]
    assert scores == sorted(scores, reverse=True)
    for r in regions[6:]:
        assert not r.p
