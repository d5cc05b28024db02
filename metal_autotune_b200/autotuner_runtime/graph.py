"""GraphWrapper: a scope whose regions are substituted inside its traced
graph instead of by a hand-written replay (the reference's
autotuner_runtime/graph.py:306-502, GraphWrapper / _make_function).

On the first call with a new signature (argument shapes, dtypes, devices and
plain values; the scope's weight shapes and dtypes) the wrapped module is
traced to an aten-level torch.fx graph with make_fx, its weights entering as
the graph's first inputs so the graph reads the module's current weights on
every call. Each rule then rewrites the graph (graph_native.rewrite): its
pattern is the region's original op sequence traced on inputs of the rule's
recorded shapes, and every occurrence becomes one call of the region's
kernel spec. A rule must replace exactly its recorded number of occurrences
(or none, where the spec's fallback predicate covers the shapes); otherwise
the certified cuts are gone and that signature runs the original module
(graph.py:447-458). Warm calls are a signature lookup and the rewritten
graph's call.

GRAPH_VARIANTS lists what the bundle recorded, one entry per call
signature it serves: {"args": [[shape, dtype], ...] of the tensor arguments,
"rules": [...]}. A call whose tensor arguments match no variant runs the
original module (graph.py:443-447).

A rule:
  kernel_id   the kernel spec that replaces the region
  sequence    "module:function" of the region's original ops
  bind        keyword constants the sequence takes (a head count, an eps)
  input_specs [[shape, dtype], ...] of the sequence's tensor inputs
  count       occurrences the rule replaces in the scope
  anchors     per input: null, ["argument", i] or ["weight", "dotted.name"]:
              that input must be that argument or weight (graph.py:478-482)
"""
from __future__ import annotations

import importlib
import os

import torch
import torch.fx as fx
import torch.nn as nn
from torch.fx.experimental.proxy_tensor import make_fx

from . import graph_native
from . import kernels as _kernels
from .swap import ReplayWrapper

GRAPH_CACHE_MAX = 64  # rewritten graphs kept per scope, one per call signature


class GraphBindingError(RuntimeError):
    """The traced graph no longer holds exactly the certified cuts."""


class RegionCall(nn.Module):
    """One region of a rewritten graph: the kernel spec's call on the
    occurrence's bound inputs, returning its boundary outputs."""

    def __init__(self, spec: _kernels.KernelSpec, n_outputs: int):
        super().__init__()
        self.spec, self.n_outputs = spec, n_outputs

    def forward(self, *inputs):
        return tuple(_kernels.call(self.spec, list(inputs))[: self.n_outputs])


def sequence_of(rule: dict):
    """The region's original-op function of a rule."""
    module, _, name = rule["sequence"].partition(":")
    fn = getattr(importlib.import_module(module), name)
    bind = dict(rule.get("bind") or {})

    def sequence(*inputs):  # positional tensor inputs only (defaults of fn stay defaults)
        return fn(*inputs, **bind)
    return sequence


def _weights(module: nn.Module) -> list[tuple[str, nn.Module, str]]:
    """(dotted name, owner, attribute) of every parameter and buffer."""
    out = []
    for prefix, sub in module.named_modules(remove_duplicate=False):
        for attr, t in list(sub._parameters.items()) + list(sub._buffers.items()):
            if t is not None:
                out.append((f"{prefix}.{attr}" if prefix else attr, sub, attr))
    seen, unique = set(), []
    for name, sub, attr in out:
        if name not in seen:
            seen.add(name)
            unique.append((name, sub, attr))
    return unique


def _sig(v):
    if isinstance(v, torch.Tensor):
        return ("tensor", tuple(v.shape), v.dtype, v.device)
    if isinstance(v, (list, tuple)):
        return (type(v).__name__, tuple(_sig(x) for x in v))
    if isinstance(v, dict):
        return ("dict", tuple((k, _sig(x)) for k, x in v.items()))
    if v is None or isinstance(v, (int, float, str, bool, torch.dtype)):
        return v
    raise GraphBindingError(f"argument of type {type(v).__name__} has no graph signature")


def trace(module: nn.Module, args: tuple, names: list[str]) -> fx.GraphModule:
    """The module's forward as an aten-level graph whose inputs are the named
    weights followed by the arguments (shapes from fake tensors: nothing is
    computed)."""
    n = len(names)

    def run(*flat):
        return torch.func.functional_call(module, dict(zip(names, flat[:n])), tuple(flat[n:]))

    current = [_resolve(module, name) for name in names]
    return make_fx(run, tracing_mode="fake")(*current, *args)


def _resolve(module, name):
    obj = module
    for part in name.split("."):
        obj = getattr(obj, part)
    return obj


class GraphWrapper(ReplayWrapper):
    """A scope served by its traced graph with the rules' regions substituted.
    Subclasses declare KERNEL_IDS and GRAPH_RULES."""

    GRAPH_VARIANTS: tuple = ()
    KERNEL_IDS: tuple = ()
    GRAPH_BACKEND = True

    def __init__(self, wrapped, specs=None):
        super().__init__(wrapped, specs)
        weights = _weights(wrapped)
        object.__setattr__(self, "_weight_slots", [(sub, attr) for _, sub, attr in weights])
        object.__setattr__(self, "_weight_names", [name for name, _, _ in weights])
        object.__setattr__(self, "_graph_functions", {})
        object.__setattr__(self, "_graph_evidence", [])   # per built signature: per-rule hits
        object.__setattr__(self, "_graph_fallbacks", [])  # why a signature runs the original

    def _live(self) -> list[torch.Tensor]:
        return [getattr(sub, attr) for sub, attr in self._weight_slots]

    def forward(self, *args):
        weights = self._live()
        key = (_sig(args), tuple((tuple(w.shape), w.dtype, w.device) for w in weights))
        entry = self._graph_functions.get(key)
        if entry is None:
            try:
                variant = self.variant_for(args)
                if variant is None:
                    raise GraphBindingError("no recorded variant for these argument shapes")
                entry = self.build_graph(args, variant["rules"])
            except GraphBindingError as problem:
                if os.environ.get("MT_STRICT_REGIONS", "0") == "1":
                    raise
                self._graph_fallbacks.append(str(problem))
                entry = False
            if len(self._graph_functions) >= GRAPH_CACHE_MAX:
                del self._graph_functions[next(iter(self._graph_functions))]
            self._graph_functions[key] = entry
        if entry is False:
            return self.wrapped(*args)
        return entry(*weights, *args)

    def variant_for(self, args: tuple) -> dict | None:
        """The recorded variant whose tensor arguments have these shapes and dtypes."""
        got = [[list(a.shape), str(a.dtype).removeprefix("torch.")] for a in args if isinstance(a, torch.Tensor)]
        for variant in self.GRAPH_VARIANTS:
            if [[list(s), d] for s, d in variant["args"]] == got:
                return variant
        return None

    def build_graph(self, args: tuple, rules) -> fx.GraphModule:
        """Trace the scope for these arguments and apply every rule; raises
        GraphBindingError when a rule's hit count is not the recorded one."""
        try:
            gm = trace(self.wrapped, args, self._weight_names)
        except Exception as problem:  # an untraceable call runs the original
            raise GraphBindingError(f"trace failed: {problem}") from problem
        device = next((a.device for a in args if isinstance(a, torch.Tensor)), torch.device("cpu"))
        n_w = len(self._weight_names)
        evidence = []
        for rule in rules:
            spec = self._specs[rule["kernel_id"]]
            inputs = [torch.empty(shape, dtype=getattr(torch, dtype), device=device)
                      for shape, dtype in rule["input_specs"]]
            pattern = make_fx(sequence_of(rule), tracing_mode="fake")(*inputs)
            n_out = len(graph_native.table(pattern).roots)
            active = not _kernels.fallback_fires(spec, inputs)
            anchors = None
            if rule.get("anchors"):
                anchors = []
                for a in rule["anchors"]:
                    if a is None:
                        anchors.append(None)
                    elif a[0] == "argument":
                        anchors.append(n_w + int(a[1]))
                    elif a[0] == "weight":
                        anchors.append(self._weight_names.index(a[1]))
                    else:
                        raise GraphBindingError(f"unknown anchor kind {a[0]!r}")

            def replace(nodes, spec=spec, n_out=n_out):
                vals = [n.meta.get("val") for n in nodes]
                if any(not isinstance(v, torch.Tensor) for v in vals) or _kernels.fallback_fires(spec, vals):
                    return None
                return RegionCall(spec, n_out)

            gm, hits = graph_native.rewrite(gm, pattern, replace, anchors)
            expected = rule["count"] if active else 0
            if hits != expected:
                raise GraphBindingError(
                    f"kernel {spec.kernel_id}: replaced {hits} graph cuts, expected {expected}; "
                    "a rule replaces every identical occurrence in its scope")
            evidence.append({"kernel_id": spec.kernel_id, "hits": hits, "expected": expected,
                             "boundary_outputs": n_out})
        self._graph_evidence.append(evidence)
        gm.recompile()
        return gm

    def regions_left(self, args: tuple) -> list[str]:
        """aten operations the rewritten graph still runs itself for these
        arguments (views and getitems aside): empty when every computing op of
        the scope is a region."""
        variant = self.variant_for(args)
        if variant is None:
            raise GraphBindingError("no recorded variant for these argument shapes")
        gm = self.build_graph(args, variant["rules"])
        light = ("view", "_unsafe_view", "reshape", "t.default", "transpose", "permute", "expand", "getitem",
                 "alias", "slice", "select", "unsqueeze", "squeeze")
        left = []
        for n in gm.graph.nodes:
            if n.op == "call_function" and not any(s in str(n.target) for s in light):
                left.append(str(n.target))
        return left
