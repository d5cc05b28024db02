"""Native graph substitution on torch.fx graphs (libmt_graph.so through
autotuner_runtime.graph_native): the behaviours the reference's
tests/test_graph_native.py pins for its MLX rewriter, on aten graphs traced
by make_fx on the CPU. Replacement regions here are small torch modules, so
every rewritten graph can be run and compared with the original."""
import ctypes

import numpy as np
import pytest
import torch
from torch.fx.experimental.proxy_tensor import make_fx

from metal_autotune_b200.autotuner_runtime import graph_native as G


def arrays(shape=(2, 3), dtype=torch.float32):
    return (torch.tensor([[1, 2, 3], [4, 5, 6]], dtype=dtype).reshape(shape),
            torch.tensor([[6, 5, 4], [3, 2, 1]], dtype=dtype).reshape(shape))


class Fn(torch.nn.Module):
    """A region standing in for a kernel: runs fn and counts its calls."""

    def __init__(self, fn):
        super().__init__()
        self.fn, self.calls = fn, 0

    def forward(self, *a):
        self.calls += 1
        out = self.fn(*a)
        return tuple(out) if isinstance(out, (list, tuple)) else (out,)


def trace(fn, *args):
    return make_fx(fn)(*args)


def run_equal(gm, fn, *args):
    got, want = gm(*args), fn(*args)
    got = got if isinstance(got, (list, tuple)) else [got]
    want = want if isinstance(want, (list, tuple)) else [want]
    assert len(got) == len(want)
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_replaces_fusion_and_preserves_internal_outside_consumer():
    pattern = trace(lambda p, q: torch.exp(p + q), *arrays())

    def model(x, y):
        shared = x + y
        return torch.exp(shared), shared * x
    gm = trace(model, *arrays())
    region = Fn(lambda a, b: torch.exp(a + b))
    new, hits = G.rewrite(gm, pattern, lambda ins: region)
    assert hits == 1
    # the outside consumer still needs the shared addition, recomputed by its original op
    assert sum(1 for n in new.graph.nodes if n.target == torch.ops.aten.add.Tensor) == 1
    assert not G.same_structure(gm, new)[0]
    run_equal(new, model, *arrays())
    assert region.calls == 1


def test_replaces_multiple_separate_boundary_outputs_together():
    pattern = trace(lambda p, q: (torch.exp(p + q), p * q), *arrays())

    def model(x, y):
        first, second = torch.exp(x + y), x * y
        return first + second, first, second
    calls = []

    def replacement(ins):
        calls.append(ins)
        return Fn(lambda a, b: (torch.exp(a + b), a * b))
    new, hits = G.rewrite(trace(model, *arrays()), pattern, replacement)
    assert hits == len(calls) == 1
    run_equal(new, model, *arrays())


def test_boundary_output_with_additional_independent_input():
    r = torch.tensor([2.0, 3.0, 4.0])
    pattern = trace(lambda p, q, r: (p + q, (p + q) * r), *arrays(), r)
    model = lambda x, y, z: (x + y, (x + y) * z)
    new, hits = G.rewrite(trace(model, *arrays(), r), pattern,
                          lambda ins: Fn(lambda a, b, c: (a + b, (a + b) * c)))
    assert hits == 1
    run_equal(new, model, *arrays(), r)


def test_live_intermediate_is_also_a_boundary_output():
    pattern = trace(lambda p, q: (p + q, torch.exp(p + q)), *arrays())

    def model(x, y):
        s = x + y
        return s, torch.exp(s)
    new, hits = G.rewrite(trace(model, *arrays()), pattern, lambda ins: Fn(lambda a, b: (a + b, torch.exp(a + b))))
    # the pattern traced p + q twice; the model computes it once: a different sharing, so no match
    assert hits == 0

    def pattern_fn(p, q):
        s = p + q
        return s, torch.exp(s)
    new, hits = G.rewrite(trace(model, *arrays()), trace(pattern_fn, *arrays()),
                          lambda ins: Fn(lambda a, b: (a + b, torch.exp(a + b))))
    assert hits == 1
    run_equal(new, model, *arrays())


@pytest.mark.parametrize("kind", ["shape", "dtype", "operator", "axis", "alias", "scalar"])
def test_nonmatching_case_is_untouched(kind):
    x, y = arrays()
    fn, args, pfn, pargs = (lambda a, b: a + b), (x, y), (lambda p, q: p + q), arrays()
    if kind == "shape":
        args = (x.t().contiguous(), y.t().contiguous())
    elif kind == "dtype":
        args = (x.half(), y.half())
    elif kind == "operator":
        fn = lambda a, b: a - b
    elif kind == "axis":
        fn, args = (lambda a: a.sum(1)), (x.t().contiguous(),)
        pfn, pargs = (lambda p: p.sum(0)), (x,)
    elif kind == "alias":
        pfn, pargs = (lambda p: p + p), (x,)
    elif kind == "scalar":
        fn, args = (lambda a: a + 2), (x,)
        pfn, pargs = (lambda p: p + 1), (x,)
    gm = trace(fn, *args)
    new, hits = G.rewrite(gm, trace(pfn, *pargs), lambda ins: pytest.fail("unexpected match"))
    assert hits == 0
    assert new is gm


def test_scalar_constants_match_without_becoming_wildcards():
    x, _ = arrays()
    model = lambda a: (a + 1, a + 2)
    new, hits = G.rewrite(trace(model, x), trace(lambda p: p + 1, x), lambda ins: Fn(lambda a: a + 1))
    assert hits == 1
    run_equal(new, model, x)


def test_callback_can_decline_specific_live_inputs():
    x, y = arrays()
    model = lambda a, b, c: (a + b, c + b)
    gm = trace(model, x, y, x.clone())
    seen = []

    def replacement(ins):
        seen.append(ins[0].name)
        return Fn(lambda a, b: a + b) if ins[0].name == "a_1" else None
    new, hits = G.rewrite(gm, trace(lambda p, q: p + q, x, y), replacement)
    assert hits == 1 and len(seen) == 2
    run_equal(new, model, x, y, x.clone())


def test_downstream_multioutput_op_keeps_every_sibling():
    x, y = arrays(shape=(3, 2))
    model = lambda a, b: tuple(torch.linalg.qr(a + b))
    new, hits = G.rewrite(trace(model, x, y), trace(lambda p, q: p + q, x, y), lambda ins: Fn(lambda a, b: a + b))
    assert hits == 1
    run_equal(new, model, x, y)


def test_multioutput_op_inside_a_pattern_binds_siblings_together():
    x, y = arrays(shape=(3, 2))
    pattern = trace(lambda p: tuple(torch.linalg.qr(p)), x)
    # both outputs of one qr call form one occurrence; an occurrence never
    # takes its outputs from two separate calls (make_fx keeps a getitem node
    # for every output of each call, so each call is a complete occurrence)
    one = trace(lambda a: tuple(torch.linalg.qr(a)), x)
    model = lambda a, b: (torch.linalg.qr(a)[0], torch.linalg.qr(b)[1])
    two = trace(model, x, y)
    region = lambda ins: Fn(lambda a: tuple(torch.linalg.qr(a)))
    assert G.rewrite(one, pattern, region)[1] == 1
    gt, pt = G.table(two), G.table(pattern)
    occs = G.find(gt, pt)
    assert len(occs) == 2
    for o in occs:
        sources = {gt.nodes[i].args[0] for i in o.outputs}
        assert len(sources) == 1
    new, hits = G.rewrite(two, pattern, region)
    assert hits == 2
    run_equal(new, model, x, y)


@pytest.mark.parametrize("reverse", [False, True])
def test_parallel_projections_match_weight_anchors(reverse):
    x = torch.ones(8, 64)
    ws = [torch.full((64, 16), v) for v in (1.0, 2.0, 3.0)]
    pair = lambda a, w0, w1: (a @ w0, a @ w1)

    def model(a, w0, w1, w2):
        first, second = pair(a, w0, w1)
        roots = [first, a @ w2, second, first + second]
        return tuple(roots[::-1] if reverse else roots)
    gm = trace(model, x, *ws)
    calls = []

    def replace(ins):
        calls.append([n.name for n in ins])
        return Fn(pair)
    # anchors: the pair's weights are the model's first two weight inputs (placeholders 1 and 2)
    new, hits = G.rewrite(gm, trace(pair, x, ws[0], ws[1]), replace, anchors=[None, 1, 2])
    assert hits == len(calls) == 1
    assert calls[0] == ["a_1", "w0_1", "w1_1"]
    run_equal(new, model, x, *ws)


def test_parallel_pattern_cannot_use_one_operation_twice():
    x, y = arrays()
    pattern = trace(lambda p, q: (p + q, p + q), x, y)
    gm = trace(lambda a, b: a + b, x, y)
    new, hits = G.rewrite(gm, pattern, lambda ins: Fn(lambda a, b: (a + b, a + b)))
    assert hits == 0


def test_anchored_boundary_parameters_can_alias():
    x, _ = arrays()
    model = lambda a: a + a
    new, hits = G.rewrite(trace(model, x), trace(lambda p, q: p + q, x, x.clone()), lambda ins: Fn(lambda a, b: a + b),
                          anchors=[0, 0])
    assert hits == 1
    run_equal(new, model, x)


def test_replacement_that_would_make_a_cycle_is_refused():
    x, y = arrays()

    def model(a, b):
        y1 = a + b
        z = y1 * 2
        return y1, torch.exp(z)
    pattern = trace(lambda p, q, r: (p + q, torch.exp(r)), x, y, x.clone())  # distinct tensors: make_fx aliases repeats
    with pytest.raises(G.GraphError, match="cycle"):
        G.rewrite(trace(model, x, y), pattern, lambda ins: Fn(lambda a, b, c: (a + b, torch.exp(c))))


def test_same_structure_and_same_computation():
    x, y = arrays()
    fn = lambda a, b: torch.exp(a + b) * a
    assert G.same_structure(trace(fn, x, y), trace(fn, x, y))[0]
    other = lambda a, b: torch.exp(a + b) * b
    same, why = G.same_structure(trace(fn, x, y), trace(other, x, y))
    assert not same and why

    def with_const(a):
        return a * torch.tensor([1.0, 2.0, 3.0])
    g1, g2 = trace(with_const, x), trace(with_const, x)
    # constants remade on each trace: different objects, same bytes
    assert not G.same_structure(g1, g2)[0]
    assert G.same_computation(g1, g2)[0]
    g3 = trace(lambda a: a * torch.tensor([1.0, 2.0, 4.0]), x)
    assert not G.same_computation(g1, g3)[0]


def test_same_structure_sees_sharing():
    x, _ = arrays()

    def shared(a):
        s = torch.exp(a)
        return s + s

    def separate(a):
        return torch.exp(a) + torch.exp(a)
    same, why = G.same_structure(trace(shared, x), trace(separate, x))
    assert not same and ("merged" in why or "duplicated" in why)


def test_engine_rejects_a_table_out_of_topological_order():
    lib = G._lib()
    op = np.array([0, 5], np.int64)
    typ = np.array([1, 1], np.int64)
    leaf = np.array([1, 0], np.int64)
    off = np.array([0, 1, 2], np.int32)
    idx = np.array([1, 0], np.int32)  # node 0 reads node 1: not topological
    view = G._View(2, op.ctypes.data, typ.ctypes.data, leaf.ctypes.data, off.ctypes.data, idx.ctypes.data)
    roots = np.array([1], np.int32)
    buf = (ctypes.c_int32 * 8)()
    rc = lib.mt_graph_order(ctypes.byref(view), roots.ctypes.data, 1, None, 0, 0, 1, None, buf, 4)
    assert rc == -1
    assert b"precede" in lib.mt_graph_error_string()
    assert lib.mt_graph_version() == 1


def test_header_declares_every_exported_symbol():
    from pathlib import Path
    import re
    header = (Path(__file__).resolve().parents[1] / "include" / "mt_graph.h").read_text()
    names = set(re.findall(r"\b(mt_graph_\w+)\s*\(", header))
    assert names == {"mt_graph_find", "mt_graph_order", "mt_graph_same", "mt_graph_error_string", "mt_graph_version"}
    lib = G._lib()
    for name in names:
        assert hasattr(lib, name)
