"""The verification ladder on the GPU: the Qwen3 RMSNorm region kernel climbs
every gate, and each cheat of the zoo dies at exactly the gate the
reference's cheat map names (tests/cheats/__init__.py:237-247)."""
from __future__ import annotations

import pytest
import torch

import ladder_cheats as Z
from metal_autotune_b200 import ladder as L

pytestmark = pytest.mark.gpu

ALL = list(L.GATES)


def _climb(job):
    res = L.run_ladder(job)
    return res


def test_region_kernel_passes_every_gate(cuda):
    res = _climb(Z.rms_norm_job(Z.rms_norm_spec(), "cuda"))
    assert res.passed, (res.failed_gate, res.detail)
    assert res.gates_passed == ALL
    assert res.info["correctness_rule"] == "tolerance"
    assert res.info["regime_magnitude"]["outliers"] == L.OUTLIER_VALUE
    assert res.info["fallback_engaged"] == {"rows256": False, "rows3": False}
    assert res.info["timing"]["candidate_ms"] > 0


def test_torch_restatement_passes_exactly(cuda):
    """The original's own ops as a stand-in: bit for bit on every gate; the
    watchdog is recorded as skipped, not passed."""
    res = _climb(Z.LadderJob(lambda inputs, init: Z.rms_norm_original(inputs), Z.rms_norm_original,
                             Z.rms_norm_job(None, "cuda").contract, Z.rms_norm_sets("cuda"),
                             weights=(False, True), exact=True))
    assert res.passed, (res.failed_gate, res.detail)
    assert res.gates_passed == [g for g in ALL if g != "watchdog"]
    assert "skipped" in res.info["watchdog"]


@pytest.mark.parametrize("builder", [Z.partial_write, Z.shape_hardcoded, Z.stride_lying, Z.eps_dropping,
                                     Z.fallback_declared_but_dead])
def test_spec_cheat_dies_at_its_gate(cuda, builder):
    spec, gate, why = builder()
    res = _climb(Z.rms_norm_job(spec, "cuda"))
    assert not res.passed, why
    assert res.failed_gate == gate, (why, res.failed_gate, res.detail)
    assert res.gates_passed == ALL[:ALL.index(gate)]


def test_cheat_details_name_what_went_wrong(cuda):
    res = _climb(Z.rms_norm_job(Z.partial_write()[0], "cuda"))
    assert res.detail["non_finite_over_finite_ref"]["out0"] == (Z.ROWS - Z.ROWS // 2) * Z.DIM
    res = _climb(Z.rms_norm_job(Z.eps_dropping()[0], "cuda"))
    assert res.detail["kind"] == "regime" and res.detail["regime"] == "scaled_down"
    res = _climb(Z.rms_norm_job(Z.stride_lying()[0], "cuda"))
    assert res.detail["kind"] == "transposed_layout"
    res = _climb(Z.rms_norm_job(Z.shape_hardcoded()[0], "cuda"))
    assert res.detail["eval_set"] == "rows256" and "fallback_declared_but_dead" not in res.detail
    res = _climb(Z.rms_norm_job(Z.fallback_declared_but_dead()[0], "cuda"))
    assert res.detail["fallback_declared_but_dead"] is True
    assert res.detail["fallback_engaged"]["rows256"] is False


def test_fallback_missing_dies_at_static(cuda):
    spec, gate, why = Z.fallback_missing()
    res = _climb(Z.rms_norm_job(spec, "cuda", requires_fallback=True))
    assert res.failed_gate == gate == "static" and res.gates_passed == []
    assert [f["check"] for f in res.detail["failures"]] == ["fallback_missing"]


def test_live_output_dropping_dies_at_static(cuda):
    spec, gate, why = Z.live_output_dropping()
    g = torch.Generator().manual_seed(5)
    x, r = (torch.randn(Z.ROWS, Z.DIM, generator=g).bfloat16().cuda() for _ in range(2))
    w = torch.ones(Z.DIM, dtype=torch.bfloat16, device="cuda")
    contract = L.RegionContract.traced(Z.add_rms_norm_original, [x, r, w])
    res = _climb(L.LadderJob(spec, Z.add_rms_norm_original, contract, [L.EvalSet("primary", [[x, r, w]])]))
    assert res.failed_gate == gate == "static"
    assert "live_output_dropped" in [f["check"] for f in res.detail["failures"]]


def test_stand_in_dropping_an_output_dies_at_static(cuda):
    g = torch.Generator().manual_seed(6)
    x, r = (torch.randn(8, 256, generator=g).cuda() for _ in range(2))
    w = torch.ones(256, device="cuda")
    contract = L.RegionContract.traced(Z.add_rms_norm_original, [x, r, w])
    res = _climb(L.LadderJob(lambda inputs, init: Z.add_rms_norm_original(inputs)[1:], Z.add_rms_norm_original,
                             contract, [L.EvalSet("primary", [[x, r, w]])]))
    assert res.failed_gate == "static" and res.gates_passed == []


def test_cached_by_shape_dies_at_smoke(cuda):
    job = Z.rms_norm_job(None, "cuda")
    stored = Z.rms_norm_original(job.eval_sets[0].input_sets[0])[0]
    job.candidate, gate, why = Z.cached_by_shape(stored)
    job.exact = True
    res = _climb(job)
    assert res.failed_gate == gate == "smoke", (why, res.detail)
    assert res.detail["input_set"] == 1 and res.detail["kind"] == "input_set"


def test_fp16_sloppy_accumulation_dies_at_smoke(cuda):
    cand, gate, why = Z.fp16_sloppy_accumulation()
    res = _climb(Z.fp16_sum_job(cand, "cuda"))
    assert res.failed_gate == gate == "smoke", (why, res.detail)
    assert res.detail["reason"] == "tolerance" and res.detail["input_set"] == 0


def test_atomic_racy_dies_at_determinism(cuda):
    cand, gate, why = Z.atomic_racy()
    res = _climb(Z.atomic_sum_job(cand, "cuda"))
    assert res.failed_gate == gate == "determinism", (why, res.detail)
    assert res.gates_passed == [g for g in ALL if g not in ("watchdog", "determinism")]
    assert res.detail["nondeterministic_output"] == "out0"


def test_an_original_that_does_not_repeat_fails_before_any_gate(cuda):
    cand, _, _ = Z.atomic_racy()
    job = Z.atomic_sum_job(cand, "cuda")
    job.original = lambda inputs: cand(inputs, None)
    res = _climb(job)
    assert res.failed_gate == "determinism" and res.gates_passed == []
    assert "repeatable" in res.detail["reason"]


@pytest.mark.parametrize("name", list(Z.ZOO))
def test_zoo_map_every_entry_stops_at_its_gate(cuda, name):
    """The zoo as a map (the reference's CHEATS dict): every entry climbs to
    exactly the gate it names, the correct kernel to the top."""
    gate = Z.ZOO[name][1]
    res = _climb(Z.zoo_job(name))
    assert res.failed_gate == gate, (name, res.detail)
    assert res.passed == (gate is None)
    if gate is not None:
        assert gate not in res.gates_passed


def test_qwen3_gate_up_kernel_climbs_every_gate(cuda):
    """The hot path's heaviest region (gate/up projections + SwiGLU, 4-bit
    g64, Qwen3-4B widths) through the ladder against its original ops
    (MLX-affine dequantisation, two matmuls, SwiGLU with each op rounded):
    prefill and decode sizes, the qmv dispatch at one row and a ragged row
    count in the sweep."""
    from metal_autotune_b200 import workload
    from metal_autotune_b200.bundles import qwen3_specs
    from metal_autotune_b200.targets import qwen3

    spec = next(s for s in qwen3_specs() if s.kernel_id == "gate_up_swiglu")
    g = torch.Generator(device="cuda").manual_seed(3)
    wg = workload.random_quantized(9728, 2560, generator=g)
    wu = workload.random_quantized(9728, 2560, generator=g)

    def original(inputs):
        x, gw, gs, gb, uw, us, ub = inputs
        gate = torch.matmul(x, workload.dequantize(gw, gs, gb, 64, 4).t())
        up = torch.matmul(x, workload.dequantize(uw, us, ub, 64, 4).t())
        return [qwen3._swiglu(gate, up)]

    def inputs(rows, seed):
        x = torch.randn(rows, 2560, generator=torch.Generator().manual_seed(seed)).bfloat16().cuda()
        return [x, *wg, *wu]

    sets = [L.EvalSet("prefill128", [inputs(128, 0), inputs(128, 1)]),
            L.EvalSet("rows16", [inputs(16, 2)]),
            L.EvalSet("rows300", [inputs(300, 3)], correctness_only=True),
            L.EvalSet("decode1", [inputs(1, 4)], correctness_only=True)]
    contract = L.RegionContract.traced(original, sets[0].input_sets[0])
    res = _climb(L.LadderJob(spec, original, contract, sets, weights=(False,) + (True,) * 6, clock=True))
    assert res.passed, (res.failed_gate, res.detail)
    assert res.gates_passed == ALL + [L.CLOCK_GATE]
    # one fused launch against dequantising 50 M weights and two GEMMs: a resolved win
    assert res.info["ship"] is True, res.info["timing"]
    assert res.info["timing"]["candidate_ms"] < res.info["timing"]["original_ms"]


def test_clock_gate_scores_a_passing_candidate(cuda):
    """The scoring phase: after determinism the clock gate times the original
    and the candidate as interleaved loops over the primary set's input sets
    and records the ship decision (both arms are launch-bound at this size, so
    the decision itself is not asserted here)."""
    job = Z.rms_norm_job(Z.rms_norm_spec(), "cuda")
    job.clock = True
    res = _climb(job)
    assert res.passed and res.gates_passed == ALL + [L.CLOCK_GATE], res.detail
    t = res.info["timing"]
    assert t["clock_sets"] == 2 and t["clock_deltas"] == L.CLOCK_PAIRS
    assert t["region_ms"] > 0 and t["library_ms"] > 0 and t["clock_iters"] >= 1
    assert isinstance(res.info["ship"], bool) and res.info["margin_ms"] > 0
