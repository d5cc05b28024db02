"""Generate the golden fixtures of this directory from the reference's tests.

The reference (shivamg05/metal-autotune) stores no golden outputs; its
known-answer cases live as literals inside its test sources. This script
reads those sources as text (ast; nothing of the reference is imported or
run — its tests need MLX on an Apple GPU) and writes the cases as JSON:

  numeric_contract.json  tests/test_numeric_contract.py parametrize tables,
                         plus the literal cases of tests/test_ladder_numeric.py:
                         178-258 (compare / max_abs_diff known answers)
  grammar.json           tests/test_runtime.py:10-33 (launch grammar values,
                         rejections, runtime bounds)

Usage: python tests/golden/make_golden.py <reference_root>   (or MT_REFERENCE_ROOT=<reference_root>)
"""
from __future__ import annotations

import ast
import json
import os
import math
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _literal(node):
    """Evaluate a literal node, allowing 2**k, float('nan'/'inf'), unary minus."""
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        return -_literal(node.operand)
    if isinstance(node, ast.BinOp):
        a, b = _literal(node.left), _literal(node.right)
        ops = {ast.Pow: lambda: a ** b, ast.Add: lambda: a + b, ast.Sub: lambda: a - b, ast.Mult: lambda: a * b}
        return ops[type(node.op)]()
    if isinstance(node, (ast.Tuple, ast.List)):
        return [_literal(e) for e in node.elts]
    if isinstance(node, ast.Call) and isinstance(node.func, ast.Name) and node.func.id == "float":
        return float(_literal(node.args[0]))
    if isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id == "mx":
        return "mx." + node.attr  # a dtype name such as mx.int32
    raise ValueError(f"not a literal: {ast.dump(node)[:80]}")


def _parametrize(tree: ast.Module, func: str):
    for fn in ast.walk(tree):
        if isinstance(fn, ast.FunctionDef) and fn.name == func:
            for dec in fn.decorator_list:
                if isinstance(dec, ast.Call) and getattr(dec.func, "attr", "") == "parametrize":
                    names = [n.strip() for n in _literal(dec.args[0]).split(",")]
                    rows = _literal(dec.args[1])
                    return names, rows, fn.lineno
    raise KeyError(func)


def _jsonable(v):
    if isinstance(v, float) and not math.isfinite(v):
        return {"float": repr(v)}
    if isinstance(v, list):
        return [_jsonable(x) for x in v]
    return v


def numeric_contract(ref: Path) -> dict:
    src = ref / "tests" / "test_numeric_contract.py"
    tree = ast.parse(src.read_text())
    out = {"source": "tests/test_numeric_contract.py", "cases": {}}
    for func in ("test_nonfloating_corruption_is_rejected_by_every_output_gate",
                 "test_matching_nonfloating_outputs_pass",
                 "test_shared_policy_exact_and_tolerance",
                 "test_shared_policy_rejects_invalid_tolerances",
                 "test_unrepresentable_tolerances_cannot_overflow_into_a_silent_pass"):
        names, rows, line = _parametrize(tree, func)
        out["cases"][func] = {"line": line, "names": names, "rows": _jsonable(rows)}
    # literal bodies (same file): see the line numbers for the statements
    out["cases"]["test_tolerance_cannot_hide_extreme_subtraction_overflow"] = {
        "reference": [3e38], "candidate": [-3e38], "dtype": "float32",
        "expect": [{"rtol": 1.5, "atol": 0.0, "passed": False}, {"rtol": 2.5, "atol": 0.0, "passed": True}]}
    out["cases"]["test_output_defaults_follow_each_dtype"] = {
        "defaults": {"float16": [1e-2, 2e-2], "float32": [1e-5, 1e-6]}, "override": [0.01, 0.0001]}
    out["cases"]["test_exact_mismatch_has_no_fictitious_numeric_distance"] = {
        "candidate": [1.0], "reference": [2.0], "reason": "exact", "max_excess": None}
    out["cases"]["test_largest_finite_tolerance_still_obeys_zero_reference_rule"] = {
        "candidate": [1.0], "reference": [0.0], "rtol": "MAX_TOLERANCE", "atol": 0.0, "passed": False}
    # tests/test_ladder_numeric.py: deterministic known answers
    out["ladder"] = {
        "source": "tests/test_ladder_numeric.py",
        "within_tolerance": {"reference": [1.0] * 4, "candidate": [1.05] * 4, "rtol": 0.0, "atol": 0.1,
                             "passed": True},
        "worst_offender": {"reference": [[1.0] * 3] * 2, "candidate": [[1.0, 1.0, 1.0], [1.0, 1.0, 1.5]],
                           "rtol": 0.0, "atol": 0.1, "passed": False, "reason": "tolerance", "index": [1, 2],
                           "max_excess": 0.4},
        "wobble_rescues": {"reference": [[1.0] * 3] * 2, "candidate": [[1.0, 1.0, 1.0], [1.0, 1.0, 1.5]],
                           "rtol": 0.0, "atol": 0.1, "wobble": 0.6, "passed": True},
        "candidate_nonfinite": {"reference": [[1.0] * 3] * 2,
                                "candidate": [[1.0, {"float": "nan"}, 1.0], [1.0, 1.0, {"float": "inf"}]],
                                "rtol": 1.0, "atol": 1e6, "passed": False, "reason": "nonfinite_pattern",
                                "index": [0, 1]},
        "reference_nonfinite_same": {
            "reference": [1.0, {"float": "nan"}, {"float": "inf"}, {"float": "-inf"}],
            "candidate": [1.0, {"float": "nan"}, {"float": "inf"}, {"float": "-inf"}], "passed": True},
        "reference_nonfinite_wrong_sign": {
            "reference": [1.0, {"float": "nan"}, {"float": "inf"}, {"float": "-inf"}],
            "candidate": [1.0, {"float": "nan"}, {"float": "-inf"}, {"float": "-inf"}], "passed": False,
            "reason": "nonfinite_pattern", "index": [2]},
        "reference_nonfinite_finite_for_nan": {
            "reference": [1.0, {"float": "nan"}, {"float": "inf"}, {"float": "-inf"}],
            "candidate": [1.0, 2.0, {"float": "inf"}, {"float": "-inf"}], "passed": False,
            "reason": "nonfinite_pattern", "index": [1]},
        "max_abs_diff": [
            {"a": [1.0, 2.0], "b": [1.0, 2.0], "value": 0.0},
            {"a": [1.0, 2.5], "b": [1.0, 2.0], "value": 0.5},
            {"a": [{"float": "nan"}, 2.0], "b": [{"float": "nan"}, 2.0], "value": 0.0},
            {"a": [{"float": "nan"}, 2.0], "b": [1.0, 2.0], "value": {"float": "inf"}},
        ],
    }
    return out


def grammar(ref: Path) -> dict:
    src = ref / "tests" / "test_runtime.py"
    tree = ast.parse(src.read_text())
    values = []
    for fn in ast.walk(tree):
        if isinstance(fn, ast.FunctionDef) and fn.name == "test_grammar_evaluates":
            for st in fn.body:
                # assert Expr("...").evaluate([...]) == value   |   ... is True
                t = st.test
                call, expected = t.left, _literal(t.comparators[0])
                expr = _literal(call.func.value.args[0])
                shapes = _literal(call.args[0])
                values.append({"expr": expr, "shapes": shapes, "value": expected})
    _, bad, line = _parametrize(tree, "test_grammar_rejects_everything_outside")
    return {"source": "tests/test_runtime.py", "evaluates": values, "rejects": bad, "rejects_line": line,
            "runtime_bounds": [{"expr": "in2.shape[0]", "shapes": [[4]], "match": "out of range"},
                               {"expr": "in0.shape[5]", "shapes": [[4]], "match": "axis"}]}


def main(ref_root: str | None = None) -> None:
    """Regenerate the fixtures from the reference checkout named by the first
    argument or, failing that, the MT_REFERENCE_ROOT environment variable."""
    ref_root = ref_root or os.environ.get("MT_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: make_golden.py <reference checkout>  (or set MT_REFERENCE_ROOT)")
    ref = Path(ref_root)
    (HERE / "numeric_contract.json").write_text(json.dumps(numeric_contract(ref), indent=1) + "\n")
    (HERE / "grammar.json").write_text(json.dumps(grammar(ref), indent=1) + "\n")


if __name__ == "__main__":
    main(*sys.argv[1:])
