"""Launch grammar: integer/boolean expressions over a call's input shapes.

Same language as the reference's autotuner_runtime/grammar.py:1-150 (the
region contract shares one grammar for output shapes, ABI size arguments and
fallback predicates): names in0, in1, ... with `.shape[i]` and `.ndim`;
calls min, max, ceil_div (exactly two positional arguments); operators
+ - * // % and / (integer division), unary -, not, single comparisons,
and/or; integer and boolean literals only. Anything else is a GrammarError,
raised when the expression is parsed. Out-of-range inputs or axes raise a
GrammarError when evaluated.

The text is parsed once (no eval) and compiled into nested closures, so a
launch lookup costs a few function calls per expression.
"""
from __future__ import annotations

import ast
import operator
from typing import Callable, Sequence

Shapes = Sequence[Sequence[int]]


class GrammarError(ValueError):
    """The expression is outside the launch grammar, or refers to an input or
    axis the call does not have."""


def _ceil_div(a, b):
    return -(-a // b)


_BIN = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul,
        ast.FloorDiv: operator.floordiv, ast.Div: operator.floordiv, ast.Mod: operator.mod}
_CMP = {ast.Lt: operator.lt, ast.LtE: operator.le, ast.Gt: operator.gt, ast.GtE: operator.ge,
        ast.Eq: operator.eq, ast.NotEq: operator.ne}
_FN = {"min": min, "max": max, "ceil_div": _ceil_div}


def _input_of(node: ast.AST, text: str) -> int:
    if isinstance(node, ast.Name) and node.id.startswith("in") and node.id[2:].isdigit():
        return int(node.id[2:])
    raise GrammarError(f"{text!r}: inputs are named in0, in1, ...")


def _compile(node: ast.AST, text: str) -> Callable[[Shapes], int | bool]:
    if isinstance(node, ast.Constant):
        v = node.value
        if type(v) not in (int, bool):
            raise GrammarError(f"{text!r}: only integer and boolean literals")
        return lambda s: v
    if isinstance(node, ast.BinOp):
        op = _BIN.get(type(node.op))
        if op is None:
            raise GrammarError(f"{text!r}: operator {type(node.op).__name__} is outside the grammar")
        a, b = _compile(node.left, text), _compile(node.right, text)
        return lambda s: op(a(s), b(s))
    if isinstance(node, ast.UnaryOp):
        a = _compile(node.operand, text)
        if isinstance(node.op, ast.USub):
            return lambda s: -a(s)
        if isinstance(node.op, ast.Not):
            return lambda s: not a(s)
        raise GrammarError(f"{text!r}: unary {type(node.op).__name__} is outside the grammar")
    if isinstance(node, ast.Compare):
        if len(node.ops) != 1 or type(node.ops[0]) not in _CMP:
            raise GrammarError(f"{text!r}: only single binary comparisons")
        op = _CMP[type(node.ops[0])]
        a, b = _compile(node.left, text), _compile(node.comparators[0], text)
        return lambda s: op(a(s), b(s))
    if isinstance(node, ast.BoolOp):
        parts = [_compile(v, text) for v in node.values]
        if isinstance(node.op, ast.And):
            return lambda s: all(p(s) for p in parts)
        return lambda s: any(p(s) for p in parts)
    if isinstance(node, ast.Call):
        if not (isinstance(node.func, ast.Name) and node.func.id in _FN):
            raise GrammarError(f"{text!r}: only min/max/ceil_div calls")
        if node.keywords or len(node.args) != 2:
            raise GrammarError(f"{text!r}: grammar calls take exactly two positional args")
        fn = _FN[node.func.id]
        a, b = (_compile(x, text) for x in node.args)
        return lambda s: fn(a(s), b(s))
    if isinstance(node, ast.Attribute):
        if node.attr != "ndim":
            raise GrammarError(f"{text!r}: only .ndim and .shape[i] accessors")
        i = _input_of(node.value, text)

        def ndim(s):
            _has_input(i, s, text)
            return len(s[i])
        return ndim
    if isinstance(node, ast.Subscript):
        if not (isinstance(node.value, ast.Attribute) and node.value.attr == "shape"):
            raise GrammarError(f"{text!r}: only .shape[i] subscripts")
        i = _input_of(node.value.value, text)
        axis = _compile(node.slice, text)

        def dim(s):
            _has_input(i, s, text)
            ax = axis(s)
            try:
                return s[i][ax]
            except IndexError:
                raise GrammarError(f"{text!r}: axis {ax} out of range for input {i} "
                                   f"with shape {tuple(s[i])}") from None
        return dim
    raise GrammarError(f"{text!r}: {type(node).__name__} is outside the launch grammar")


def _has_input(i: int, s: Shapes, text: str) -> None:
    if i >= len(s):
        raise GrammarError(f"{text!r}: input {i} out of range, call has {len(s)} inputs")


class Expr:
    """A parsed launch-grammar expression, reusable across calls."""

    __slots__ = ("text", "_fn")

    def __init__(self, text: str):
        self.text = text
        try:
            tree = ast.parse(text, mode="eval").body
        except (SyntaxError, RecursionError, MemoryError, ValueError) as e:
            raise GrammarError(f"cannot parse {text!r}: {type(e).__name__}: {e}") from None
        try:
            self._fn = _compile(tree, text)
        except RecursionError:
            raise GrammarError(f"cannot parse {text!r}: expression too deep") from None

    def evaluate(self, shapes: Shapes) -> int | bool:
        """shapes[i] is the concrete shape of input i for this call."""
        return self._fn(shapes)

    def __repr__(self) -> str:
        return f"Expr({self.text!r})"

    def __eq__(self, other) -> bool:
        return isinstance(other, Expr) and other.text == self.text

    def __hash__(self) -> int:
        return hash(self.text)
