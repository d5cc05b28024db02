"""Certified graph substitution on torch.fx graphs, with the graph walks in
native code (libmt_graph.so, include/mt_graph.h).

The reference rewrites MLX's lazy array graph through a C++ extension
(autotuner_runtime/graph_native/__init__.py:127-141, graph_native.cpp):
`rewrite(roots, pattern_outputs, parameters, replacement, anchors)` returns
the new roots and the number of replacements, and `same_structure` /
`same_computation` prove two graphs equal. Here the graphs are aten-level
torch.fx graphs traced by make_fx (shapes and dtypes in node.meta["val"]):

  rewrite(gm, pattern, replacement, anchors=None) -> (GraphModule, hits)
      pattern: a GraphModule whose placeholders are the region's boundary
      inputs and whose outputs are its boundary outputs. replacement(inputs)
      gets the bound input nodes of one occurrence (their meta["val"] holds
      shape and dtype) and returns a module to call in its place, or None to
      keep that occurrence. The new graph calls each returned module with the
      occurrence's inputs; its outputs stand for the occurrence's outputs
      everywhere they were used. Nodes nothing uses any more are dropped; a
      value an outside consumer still reads from inside an occurrence stays
      computed by its original ops (graph_native.cpp:180-259).
  same_structure(a, b) / same_computation(b) -> (bool, reason)
      same operations, attributes, leaves and sharing from the outputs; a
      constant (get_attr) leaf is the same object, or, for same_computation,
      the same shape, dtype and bytes (graph_native.cpp:261-322).

Operation keys are the aten overload with every non-tensor argument (so
`x + 1` never matches `x + 2`, graph_native.cpp:53-58); a node's type is its
value's shape and dtype. Placeholders are leaves named by position.
"""
from __future__ import annotations

import copy
import ctypes
import operator
from dataclasses import dataclass, field
from typing import Callable

import numpy as np
import torch
import torch.fx as fx

_LIB = None


class _View(ctypes.Structure):
    _fields_ = [("n_nodes", ctypes.c_int32), ("op", ctypes.c_void_p), ("type", ctypes.c_void_p),
                ("leaf", ctypes.c_void_p), ("in_off", ctypes.c_void_p), ("in_idx", ctypes.c_void_p)]


def _lib():
    """libmt_graph.so, built on first use when missing or stale."""
    global _LIB
    if _LIB is None:
        from metal_autotune_b200 import build
        lib = ctypes.CDLL(str(build.build_graph_library()))
        i32p, vp = ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p
        lib.mt_graph_find.argtypes = [ctypes.POINTER(_View), ctypes.POINTER(_View), vp, ctypes.c_int32, vp,
                                      ctypes.c_int32, vp, i32p, ctypes.c_int32]
        lib.mt_graph_order.argtypes = [ctypes.POINTER(_View), vp, ctypes.c_int32, vp, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int32, vp, i32p, ctypes.c_int32]
        lib.mt_graph_same.argtypes = [ctypes.POINTER(_View), vp, ctypes.POINTER(_View), vp, ctypes.c_int32,
                                      ctypes.c_char_p, ctypes.c_int32]
        lib.mt_graph_error_string.restype = ctypes.c_char_p
        for name in ("mt_graph_find", "mt_graph_order", "mt_graph_same", "mt_graph_version"):
            getattr(lib, name).restype = ctypes.c_int
        _LIB = lib
    return _LIB


class GraphError(RuntimeError):
    """The native engine refused a table or a replacement."""


def _check(rc: int, what: str) -> int:
    if rc < 0:
        raise GraphError(f"{what}: {_lib().mt_graph_error_string().decode()} (code {rc})")
    return rc


# ------------------------------------------------------------------ keys
_KEYS: dict[str, int] = {}


def _intern(text: str) -> int:
    k = _KEYS.get(text)
    if k is None:
        k = _KEYS[text] = len(_KEYS) + 1
    return k


def _sig(v) -> str:
    """A non-tensor argument or a node's value, as key text."""
    if isinstance(v, fx.Node):
        return "%"
    if isinstance(v, torch.Tensor):
        return f"T{tuple(v.shape)}:{v.dtype}"
    if isinstance(v, (list, tuple)):
        return ("[" if isinstance(v, list) else "(") + ",".join(_sig(x) for x in v) + ("]" if isinstance(v, list) else ")")
    if isinstance(v, dict):
        return "{" + ",".join(f"{k}={_sig(x)}" for k, x in v.items()) + "}"
    if isinstance(v, float):
        return repr(v) + "f"
    if isinstance(v, (torch.SymInt, torch.SymFloat)):
        return f"sym:{v}"
    return repr(v)


def _target(node: fx.Node) -> str:
    t = node.target
    if isinstance(t, str):
        return f"{node.op}:{t}"
    name = getattr(t, "__qualname__", None) or getattr(t, "__name__", None) or str(t)
    if isinstance(t, torch._ops.OpOverload):
        name = str(t)
    return f"{node.op}:{getattr(t, '__module__', '')}.{name}"


def _tensor_inputs(node: fx.Node) -> list[fx.Node]:
    ins: list[fx.Node] = []
    fx.node.map_arg((node.args, node.kwargs), lambda n: ins.append(n))
    return ins


@dataclass
class Table:
    """A torch.fx graph as the engine's node table (outputs excluded)."""
    nodes: list
    index: dict
    op: np.ndarray
    type: np.ndarray
    leaf: np.ndarray
    in_off: np.ndarray
    in_idx: np.ndarray
    roots: list
    out_node: fx.Node | None = None
    _keep: list = field(default_factory=list)

    def view(self) -> _View:
        arrs = [np.ascontiguousarray(a) for a in (self.op, self.type, self.leaf, self.in_off, self.in_idx)]
        self._keep = arrs
        ptr = lambda a: a.ctypes.data if a.size else None
        return _View(len(self.nodes), *(ptr(a) for a in arrs))


def table(gm: fx.GraphModule | fx.Graph, leaves: str = "object") -> Table:
    """Flatten a graph. leaves: "object" (a get_attr constant is its tensor
    object) or "value" (its shape, dtype and bytes)."""
    graph = gm.graph if isinstance(gm, fx.GraphModule) else gm
    owner = gm if isinstance(gm, fx.GraphModule) else None
    nodes, index = [], {}
    op, typ, leaf, off, idx = [], [], [], [0], []
    out_node, roots = None, []
    n_ph = 0
    for node in graph.nodes:
        if node.op == "output":
            out_node = node
            continue
        index[node] = len(nodes)
        nodes.append(node)
        typ.append(_intern("type " + _sig(node.meta.get("val", None))))
        if node.op == "placeholder":
            op.append(0)
            leaf.append(_intern(f"placeholder {n_ph}"))
            n_ph += 1
        elif node.op == "get_attr":
            op.append(0)
            value = _attr(owner, node.target) if owner is not None else None
            if leaves == "value" and isinstance(value, torch.Tensor):
                data = value.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()
                leaf.append(_intern(f"const {tuple(value.shape)} {value.dtype} {hash(data)} {len(data)}"))
            else:
                leaf.append(_intern(f"object {id(value) if value is not None else node.target}"))
        else:
            op.append(_intern(f"{_target(node)}|{_sig(node.args)}|{_sig(node.kwargs)}"))
            leaf.append(0)
        for n in _tensor_inputs(node):
            idx.append(index[n])
        off.append(len(idx))
    if out_node is not None:
        fx.node.map_arg(out_node.args, lambda n: roots.append(index[n]))
    return Table(nodes, index, np.asarray(op, np.int64), np.asarray(typ, np.int64), np.asarray(leaf, np.int64),
                 np.asarray(off, np.int32), np.asarray(idx, np.int32), roots, out_node)


def _attr(gm, target: str):
    obj = gm
    for part in target.split("."):
        obj = getattr(obj, part)
    return obj


def _arr(xs) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(xs), np.int32))


# ------------------------------------------------------------------ engine calls
@dataclass
class Occurrence:
    inputs: list   # bound graph node indices, one per pattern parameter
    outputs: list  # bound graph node indices, one per pattern output


def find(graph: Table, pattern: Table, anchors: list[int | None] | None = None) -> list[Occurrence]:
    """Every non-overlapping occurrence of the pattern (its placeholders are
    the parameters, its outputs the boundary outputs), in graph order."""
    params = [i for i, n in enumerate(pattern.nodes) if n.op == "placeholder"]
    outs = list(pattern.roots)
    if anchors is not None and len(anchors) != len(params):
        raise GraphError("graph anchors must align with parameters")
    anc = None if anchors is None else _arr(-1 if a is None else a for a in anchors)
    gv, pv = graph.view(), pattern.view()
    pa, oa = _arr(params), _arr(outs)
    width = len(params) + len(outs)
    cap = 16
    while True:
        buf = (ctypes.c_int32 * max(1, cap * width))()
        n = _check(_lib().mt_graph_find(ctypes.byref(gv), ctypes.byref(pv), pa.ctypes.data if pa.size else None,
                                        len(params), oa.ctypes.data, len(outs),
                                        None if anc is None else anc.ctypes.data, buf, cap), "find")
        if n <= cap:
            break
        cap = n
    flat = list(buf)[: n * width]
    return [Occurrence(flat[k * width:k * width + len(params)], flat[k * width + len(params):(k + 1) * width])
            for k in range(n)]


def order(graph: Table, occs: list[Occurrence], accept: list[bool]) -> list[tuple[int, int]]:
    """The rewritten graph's nodes in a valid order: (0, graph node) or (1, occurrence)."""
    n_params = len(occs[0].inputs) if occs else 0
    n_outs = len(occs[0].outputs) if occs else 1
    occ = _arr(x for o in occs for x in (*o.inputs, *o.outputs))
    acc = np.ascontiguousarray(np.asarray(accept, np.uint8))
    roots = _arr(graph.roots)
    gv = graph.view()
    cap = len(graph.nodes) + len(occs)
    buf = (ctypes.c_int32 * max(2, 2 * cap))()
    n = _check(_lib().mt_graph_order(ctypes.byref(gv), roots.ctypes.data if roots.size else None, len(graph.roots),
                                     occ.ctypes.data if occ.size else None, len(occs), n_params, n_outs,
                                     acc.ctypes.data if acc.size else None, buf, cap), "rewrite")
    flat = list(buf)[: 2 * n]
    return [(flat[2 * i], flat[2 * i + 1]) for i in range(n)]


def _same(a: Table, b: Table) -> tuple[bool, str]:
    if len(a.roots) != len(b.roots):
        return False, "root count"
    av, bv = a.view(), b.view()
    ra, rb = _arr(a.roots), _arr(b.roots)
    reason = ctypes.create_string_buffer(256)
    rc = _check(_lib().mt_graph_same(ctypes.byref(av), ra.ctypes.data if ra.size else None, ctypes.byref(bv),
                                     rb.ctypes.data if rb.size else None, len(a.roots), reason, 256), "same")
    return rc == 1, reason.value.decode()


def same_structure(a: fx.GraphModule, b: fx.GraphModule) -> tuple[bool, str]:
    """Same operations, attributes, leaves (constants by object) and sharing."""
    return _same(table(a, "object"), table(b, "object"))


def same_computation(a: fx.GraphModule, b: fx.GraphModule) -> tuple[bool, str]:
    """same_structure with constants compared by shape, dtype and bytes: two
    traces of the same Python that remake their constants on each call."""
    return _same(table(a, "value"), table(b, "value"))


# ------------------------------------------------------------------ rewrite
def rewrite(gm: fx.GraphModule, pattern: fx.GraphModule,
            replacement: Callable[[list[fx.Node]], torch.nn.Module | None],
            anchors: list[int | None] | None = None) -> tuple[fx.GraphModule, int]:
    """Replace every occurrence of `pattern` that `replacement` accepts.
    anchors[i] (a placeholder position of gm, or None) fixes parameter i."""
    gt, pt = table(gm, "value"), table(pattern, "value")
    anchor_nodes = None
    if anchors is not None:
        phs = [i for i, n in enumerate(gt.nodes) if n.op == "placeholder"]
        anchor_nodes = [None if a is None else phs[a] for a in anchors]
    occs = find(gt, pt, anchor_nodes)
    modules = [replacement([gt.nodes[i] for i in o.inputs]) for o in occs]
    accept = [m is not None for m in modules]
    hits = sum(accept)
    if hits == 0:
        return gm, 0
    seq = order(gt, occs, accept)

    new = fx.Graph()
    new.set_codegen(copy.deepcopy(gm.graph._codegen))  # keeps the traced call's argument/result structure
    env: dict[fx.Node, fx.Node] = {}
    attrs: dict[str, object] = {}
    for node in gt.nodes:
        if node.op == "placeholder":
            env[node] = new.node_copy(node)
    n_region = 0
    existing = {name for name, _ in gm.named_children()}
    for kind, i in seq:
        if kind == 0:
            node = gt.nodes[i]
            if node.op == "placeholder":
                continue
            if node.op == "get_attr":
                attrs[node.target] = _attr(gm, node.target)
            elif node.op == "call_module":
                attrs[node.target] = _attr(gm, node.target)
            env[node] = new.node_copy(node, lambda n: env[n])
            continue
        o = occs[i]
        while f"region_{n_region}" in existing:
            n_region += 1
        name = f"region_{n_region}"
        n_region += 1
        attrs[name] = modules[i]
        call = new.call_module(name, tuple(env[gt.nodes[b]] for b in o.inputs))
        vals = tuple(gt.nodes[x].meta.get("val") for x in o.outputs)
        call.meta["val"] = vals
        for j, x in enumerate(o.outputs):
            g = new.call_function(operator.getitem, (call, j))
            g.meta = dict(gt.nodes[x].meta)
            env[gt.nodes[x]] = g
    new.output(fx.node.map_arg(gt.out_node.args[0], lambda n: env[n]))
    new.lint()
    return fx.GraphModule(attrs, new), hits
