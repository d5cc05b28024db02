"""The CPU restatement of the output contract against the reference's own
known-answer cases (tests/golden/*.json, extracted from its test sources by
tests/golden/make_golden.py). These pin the oracle that the GPU diff
reduction is checked against."""
import math

import numpy as np
import pytest

from oracle import numeric_ref as N
from tests.conftest import fval, golden

G = golden("numeric_contract.json")
CASES = G["cases"]


def arr(v, dt=np.float32):
    return np.array(fval(v), dtype=dt)


_NP = {"mx.int32": np.int32, "mx.uint32": np.uint32, "mx.int64": np.int64, "mx.uint64": np.uint64,
       "mx.bool_": np.bool_}


@pytest.mark.parametrize("dtype,value", CASES["test_nonfloating_corruption_is_rejected_by_every_output_gate"]["rows"])
def test_nonfloating_corruption_rejected(dtype, value):
    dt = _NP[dtype]
    ref = np.array([value], dtype=dt)
    bad = np.array([value + 1], dtype=dt) if dt is not np.bool_ else np.array([not value], dtype=dt)
    assert not N.compare(bad, ref, rtol=1.0, atol=100.0, floating=False)["passed"]
    assert N.max_abs_diff(ref, bad, floating=False) == math.inf


@pytest.mark.parametrize("dtype,value", CASES["test_matching_nonfloating_outputs_pass"]["rows"])
def test_matching_nonfloating_pass(dtype, value):
    ref = np.array([value], dtype=_NP[dtype])
    assert N.compare(ref.copy(), ref, rtol=0.0, atol=0.0, floating=False)["passed"]
    assert N.max_abs_diff(ref, ref.copy(), floating=False) == 0.0


@pytest.mark.parametrize("reference,candidate,exact,passed", CASES["test_shared_policy_exact_and_tolerance"]["rows"])
def test_exact_and_tolerance(reference, candidate, exact, passed):
    r = N.check(arr(candidate), arr(reference), exact=exact, rtol=0.01, atol=0.001)
    assert r["passed"] is passed


def test_subtraction_overflow_cannot_hide():
    c = CASES["test_tolerance_cannot_hide_extreme_subtraction_overflow"]
    for e in c["expect"]:
        r = N.check(arr(c["candidate"]), arr(c["reference"]), exact=False, rtol=e["rtol"], atol=e["atol"])
        assert r["passed"] is e["passed"]


@pytest.mark.parametrize("values", CASES["test_shared_policy_rejects_invalid_tolerances"]["rows"])
def test_invalid_tolerances(values):
    with pytest.raises(ValueError, match="finite non-negative"):
        N.check(arr([1.0]), arr([1.0]), exact=False, rtol=fval(values[0]), atol=fval(values[1]))


@pytest.mark.parametrize("candidate,reference,rtol,atol",
                         CASES["test_unrepresentable_tolerances_cannot_overflow_into_a_silent_pass"]["rows"])
def test_unrepresentable_tolerances(candidate, reference, rtol, atol):
    with pytest.raises(ValueError, match="fit in float32"):
        N.check(arr([candidate]), arr([reference]), exact=False, rtol=rtol, atol=atol)


def test_exact_mismatch_has_no_distance():
    c = CASES["test_exact_mismatch_has_no_fictitious_numeric_distance"]
    r = N.check(arr(c["candidate"]), arr(c["reference"]))
    assert not r["passed"] and r["reason"] == c["reason"] and r["max_excess"] is None


def test_largest_tolerance_obeys_zero_reference():
    c = CASES["test_largest_finite_tolerance_still_obeys_zero_reference_rule"]
    r = N.check(arr(c["candidate"]), arr(c["reference"]), exact=False, rtol=N.MAX_TOLERANCE, atol=0.0)
    assert r["passed"] is c["passed"]


@pytest.mark.parametrize("name", ["within_tolerance", "worst_offender", "wobble_rescues", "candidate_nonfinite",
                                  "reference_nonfinite_same", "reference_nonfinite_wrong_sign",
                                  "reference_nonfinite_finite_for_nan"])
def test_ladder_known_answers(name):
    c = G["ladder"][name]
    r = N.compare(arr(c["candidate"]), arr(c["reference"]), rtol=c.get("rtol", 0.0), atol=c.get("atol", 0.0),
                  wobble=c.get("wobble", 0.0))
    assert r["passed"] is c["passed"]
    if "reason" in c:
        assert r["reason"] == c["reason"]
    if "index" in c:
        assert tuple(int(i) for i in r["index"]) == tuple(c["index"])
    if "max_excess" in c:
        assert r["max_excess"] == pytest.approx(c["max_excess"], rel=1e-5)


@pytest.mark.parametrize("case", G["ladder"]["max_abs_diff"])
def test_ladder_max_abs_diff(case):
    assert N.max_abs_diff(arr(case["a"]), arr(case["b"])) == pytest.approx(fval(case["value"]))


def test_default_tolerances_match_reference():
    from metal_autotune_b200.autotuner_runtime.numeric import DEFAULT_TOLERANCES, tolerance_for
    c = CASES["test_output_defaults_follow_each_dtype"]
    for name, tol in c["defaults"].items():
        assert tuple(DEFAULT_TOLERANCES[name]) == tuple(tol)
    assert tolerance_for("float16", tuple(c["override"])) == tuple(c["override"])
