"""Host side of the verification ladder: gate 1's static checks on KernelSpecs
against region contracts, the value regimes and the transposed layout (the
reference's tests/test_static_checks.py and tests/test_ladder_numeric.py
test the same policies). No GPU work."""
from __future__ import annotations

from dataclasses import replace

import pytest
import torch

import ladder_cheats as Z
from metal_autotune_b200 import ladder as L


def _contract(**kw):
    sets = Z.rms_norm_sets("cpu")
    return L.RegionContract.traced(Z.rms_norm_original, sets[0].input_sets[0], **kw)


def _checks(spec, contract=None):
    return [f.check for f in L.static_check(spec, contract or _contract())]


def test_traced_contract_names_ranks_dtypes_and_shapes():
    c = _contract()
    assert c.input_names == ("in0", "in1") and c.output_names == ("out0",)
    assert c.input_ranks == (2, 1) and c.output_ranks == (2,)
    assert c.input_dtypes == ("bfloat16", "bfloat16") and c.output_dtypes == ("bfloat16",)
    assert c.input_shapes == ((Z.ROWS, Z.DIM), (Z.DIM,)) and c.output_shapes == ((Z.ROWS, Z.DIM),)
    assert c.live_outputs == ("out0",) and not c.requires_fallback


def test_the_region_spec_passes_static():
    assert L.static_check(Z.rms_norm_spec(), _contract()) == []


@pytest.mark.parametrize("builder", [Z.partial_write, Z.shape_hardcoded, Z.stride_lying, Z.eps_dropping,
                                     Z.fallback_declared_but_dead])
def test_value_cheats_pass_static_so_they_reach_their_gate(builder):
    spec, gate, _ = builder()
    assert gate != "static"
    assert L.static_check(spec, _contract()) == []


def test_live_output_dropping_fails_static():
    spec, gate, _ = Z.live_output_dropping()
    g = torch.Generator().manual_seed(0)
    x, r = torch.randn(8, 64, generator=g), torch.randn(8, 64, generator=g)
    w = torch.ones(64)
    contract = L.RegionContract.traced(Z.add_rms_norm_original, [x, r, w])
    assert contract.live_outputs == ("out0", "out1")
    assert gate == "static" and "live_output_dropped" in _checks(spec, contract)


def test_fallback_missing_fails_static_only_when_the_contract_requires_one():
    spec, gate, _ = Z.fallback_missing()
    assert gate == "static"
    assert _checks(spec, _contract(requires_fallback=True)) == ["fallback_missing"]
    assert _checks(spec, _contract()) == []
    covered = replace(spec, fallback_predicate="in0.shape[0] > 4096")
    assert _checks(covered, _contract(requires_fallback=True)) == []


def test_fallback_true_on_the_primary_workload_fails():
    spec = replace(Z.rms_norm_spec(), fallback_predicate="in0.shape[0] == 64")
    assert _checks(spec) == ["fallback_on_primary"]


def test_entry_point_checks():
    spec = Z.rms_norm_spec()
    assert _checks(replace(spec, cuda={**spec.cuda, "symbol": "mt_no_such_kernel"})) == ["entry_point"]
    assert _checks(replace(spec, cuda={**spec.cuda, "args": spec.cuda["args"][:-1]})) == ["entry_point"]
    bad_in = Z._with_arg(spec, 1, {"in": 2})
    assert _checks(bad_in) == ["entry_point"]
    bad_out = Z._with_arg(spec, 3, {"out": 1})
    assert _checks(bad_out) == ["entry_point"]
    assert _checks(replace(spec, cuda=None)) == ["entry_point"]


def test_launch_grammar_is_probed_at_the_traced_shapes():
    spec = Z.rms_norm_spec()
    assert _checks(Z._with_arg(spec, 4, {"expr": "in3.shape[0]"})) == ["launch_grammar"]
    assert _checks(Z._with_arg(spec, 4, {"expr": "in0.shape[2]"})) == ["launch_grammar"]
    assert "launch_grammar" in _checks(replace(spec, fallback_predicate="in0.shape["))


def test_output_contract_checks():
    spec = Z.rms_norm_spec()
    assert _checks(replace(spec, output_shapes=(("in0.shape[0]", "in0.shape[1] // 2"),))) == ["output_shape"]
    assert _checks(replace(spec, output_shapes=(("in0.shape[0]",),))) == ["output_rank", "output_shape"]
    assert _checks(replace(spec, output_dtypes=("float32",))) == ["output_dtype"]
    assert _checks(replace(spec, output_dtypes=("in1",))) == []          # in1 is bf16 as well
    assert "output_arity" in _checks(replace(spec, output_dtypes=()))
    assert _checks(replace(spec, output_names=("y",))) == ["output_names", "live_output_dropped"]
    assert _checks(replace(spec, output_names=("out0", "tmp0"), output_shapes=spec.output_shapes * 2,
                           output_dtypes=spec.output_dtypes * 2)) == []
    assert _checks(replace(spec, output_names=("out0", "scratch"), output_shapes=spec.output_shapes * 2,
                           output_dtypes=spec.output_dtypes * 2)) == ["output_names"]


def test_names_and_signatures():
    spec = Z.rms_norm_spec()
    assert _checks(replace(spec, name="mt rms")) == ["kernel_name"]
    assert _checks(replace(spec, input_names=("x", "w"))) == ["input_names"]
    assert _checks(replace(spec, input_signature=[[[64, 2048], "bfloat16"], [[2048], "bfloat16"]])) == \
        ["input_signature"]


def test_value_regimes_leave_weights_and_integers_alone():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(6, 5, generator=g)
    w = torch.randn(5, generator=g)
    idx = torch.arange(6)
    reg = L.value_regimes([x, w, idx], seed=3, weights=(False, True, False))
    assert set(reg) == set(L.REGIMES)
    for name in L.REGIMES:
        assert reg[name][1] is w and reg[name][2] is idx
    torch.testing.assert_close(reg["scaled_down"][0], x * L.SCALE_DOWN)
    assert int((reg["outliers"][0] == L.OUTLIER_VALUE).sum()) == L.OUTLIER_COUNT
    assert not reg["zeros"][0].any()
    nf = reg["nonfinite"][0]
    inf_rows = torch.isinf(nf).all(1).nonzero().flatten().tolist()
    nan_rows = torch.isnan(nf).all(1).nonzero().flatten().tolist()
    assert len(inf_rows) == 1 and len(nan_rows) == 1 and inf_rows != nan_rows
    assert torch.isfinite(nf).sum() == 4 * 5
    # the inputs themselves are never modified, and a seed fixes the regimes
    assert torch.isfinite(x).all()
    again = L.value_regimes([x, w, idx], seed=3, weights=(False, True, False))
    assert torch.equal(again["outliers"][0], reg["outliers"][0])
    assert torch.equal(torch.isnan(again["nonfinite"][0]), torch.isnan(nf))


def test_value_regimes_at_a_smaller_outlier_and_in_half_precision():
    x = torch.ones(4, 8, dtype=torch.float16)
    reg = L.value_regimes([x], seed=0, outlier=1e2)
    assert int((reg["outliers"][0] == 100).sum()) == L.OUTLIER_COUNT
    assert reg["scaled_down"][0].dtype == torch.float16
    one_row = L.value_regimes([torch.ones(1, 3)], seed=0)["nonfinite"][0]
    assert torch.isnan(one_row).all()          # one lane: NaN planted over the inf
    scalar = L.value_regimes([torch.tensor(2.0)], seed=0)["nonfinite"][0]
    assert torch.isnan(scalar)


def test_transposed_layout_keeps_values_and_storage_size():
    x = torch.randn(5, 7)
    w = torch.randn(7)
    (xt, wt), changed = L.transposed_layout([x, w])
    assert changed and wt is w
    assert torch.equal(xt, x) and not xt.is_contiguous() and xt.stride() == (1, 5)
    assert xt.untyped_storage().nbytes() == x.untyped_storage().nbytes()
    assert L.transposed_layout([w])[1] is False


def test_every_committed_bundle_spec_binds_its_entry_point():
    """Gate 1's entry-point check on every launch record the bundles ship:
    the symbol exists and the record binds each of its parameters (a
    workspace binds two: pointer and size)."""
    from pathlib import Path

    from metal_autotune_b200.autotuner_runtime.kernels import load_spec
    bundles = Path(L.__file__).resolve().parent / "bundles"
    paths = sorted(bundles.glob("*/kernels/*.launch.json"))
    assert paths
    for path in paths:
        spec = load_spec(path)
        kernels = [st.kernel for st in spec.stages] if spec.stages else [spec]
        for k in kernels:
            bad = [f for f in L._entry_point_failures(k, len(k.input_names), len(k.output_names), [])
                   if f.check == "entry_point"]
            assert bad == [], (path.name, bad)
