"""Host logic of the region contract (no GPU): launch grammar against the
reference's known answers, KernelSpec JSON round trips, launch resolution
and fallback predicates, stage-plan validation, module swap / apply, and the
paired statistics."""
import json
import math

import pytest
import torch
import torch.nn as nn

from metal_autotune_b200.autotuner_runtime import kernels as K
from metal_autotune_b200.autotuner_runtime import stats as S
from metal_autotune_b200.autotuner_runtime.grammar import Expr, GrammarError
from metal_autotune_b200.autotuner_runtime.kernels import KernelSpec, KernelStage, LoadedKernel
from metal_autotune_b200.autotuner_runtime import swap
from tests.conftest import golden

GR = golden("grammar.json")


@pytest.mark.parametrize("case", GR["evaluates"])
def test_grammar_known_values(case):
    assert Expr(case["expr"]).evaluate([tuple(s) for s in case["shapes"]]) == case["value"]


@pytest.mark.parametrize("bad", GR["rejects"])
def test_grammar_rejects(bad):
    with pytest.raises(GrammarError):
        Expr(bad)


@pytest.mark.parametrize("case", GR["runtime_bounds"])
def test_grammar_runtime_bounds(case):
    with pytest.raises(GrammarError, match=case["match"]):
        Expr(case["expr"]).evaluate([tuple(s) for s in case["shapes"]])


def test_grammar_resource_exhaustion_is_a_rejection():
    with pytest.raises(GrammarError):
        Expr("+".join(["in0.shape[0]"] * 40000))


def _rms_spec(**kw):
    base = dict(kernel_id="t_rms", name="mt_rms_norm", input_names=("in0", "in1"), output_names=("out0",),
                cuda={"symbol": "mt_rms_norm", "args": [
                    {"in": 0}, {"in": 1}, {"float": 1e-6}, {"out": 0}, {"expr": "in0.shape[0]"},
                    {"expr": "in0.shape[1]"}, {"dtype": "in0"}, {"stream": True}]},
                output_shapes=(("in0.shape[0]", "in0.shape[1]"),), output_dtypes=("in0",))
    base.update(kw)
    return KernelSpec(**base)


def test_spec_round_trip():
    s = _rms_spec(fallback_predicate="in0.shape[1] % 8 != 0")
    assert KernelSpec.from_json(s.to_json()) == s


def test_bundle_specs_round_trip():
    from metal_autotune_b200.bundles import qwen3_specs
    for s in qwen3_specs():
        assert KernelSpec.from_json(s.to_json()) == s


def test_launch_resolution_and_fallback():
    lk = LoadedKernel(_rms_spec(fallback_predicate="in0.shape[1] % 8 != 0"))
    x = torch.zeros(4, 12, dtype=torch.bfloat16)
    w = torch.zeros(12, dtype=torch.bfloat16)
    assert lk.fallback_fires([x, w])
    x2 = torch.zeros(4, 16, dtype=torch.bfloat16)
    launch = lk.launch([x2, torch.zeros(16, dtype=torch.bfloat16)])
    assert not launch.fallback
    assert launch.output_shapes == [(4, 16)] and launch.output_dtypes == [torch.bfloat16]
    vals = [v for k, v in launch.args if k == "val"]
    assert vals[1:] == [4, 16, 0]  # rows, dim, MT_BF16 (eps first)
    assert lk.launch([x2, torch.zeros(16, dtype=torch.bfloat16)]) is launch  # cached per signature


def test_input_signature_gates_the_kernel():
    sig = [[[2, 8], "bfloat16"], [[8], "bfloat16"]]
    lk = LoadedKernel(_rms_spec(input_signature=sig))
    assert lk.fallback_fires([torch.zeros(3, 8, dtype=torch.bfloat16), torch.zeros(8, dtype=torch.bfloat16)])
    assert not lk.fallback_fires([torch.zeros(2, 8, dtype=torch.bfloat16), torch.zeros(8, dtype=torch.bfloat16)])
    # a size-generic wrapper checked elsewhere is bounded only by the predicate
    assert not lk.launch([torch.zeros(3, 8, dtype=torch.bfloat16), torch.zeros(8, dtype=torch.bfloat16)],
                         checked_elsewhere=True).fallback


def test_unknown_symbol_rejected():
    with pytest.raises(ValueError, match="not a libmt entry point"):
        LoadedKernel(_rms_spec(cuda={"symbol": "mt_nope", "args": []}))


def test_workspace_binder_queries_the_library():
    from metal_autotune_b200.bundles import qwen3_specs
    spec = next(s for s in qwen3_specs() if s.kernel_id == "qkv_qmm")
    lk = LoadedKernel(spec)
    x = torch.zeros(128, 2560, dtype=torch.bfloat16)
    ws = [torch.zeros(n, 320, dtype=torch.int32) for n in (4096,)]
    ins = [x, ws[0], torch.zeros(4096, 40, dtype=torch.bfloat16), torch.zeros(4096, 40, dtype=torch.bfloat16),
           torch.zeros(1024, 320, dtype=torch.int32), torch.zeros(1024, 40, dtype=torch.bfloat16),
           torch.zeros(1024, 40, dtype=torch.bfloat16), torch.zeros(1024, 320, dtype=torch.int32),
           torch.zeros(1024, 40, dtype=torch.bfloat16), torch.zeros(1024, 40, dtype=torch.bfloat16)]
    launch = lk.launch(ins)
    wsz = [v for k, v in launch.args if k == "workspace"]
    assert len(wsz) == 1 and wsz[0] > 0
    assert launch.output_shapes == [(128, 4096), (128, 1024), (128, 1024)]


def _stage_spec(stages, outputs=("out0",)):
    return KernelSpec(kernel_id="staged", name="staged", input_names=("in0", "in1"), output_names=outputs,
                      output_shapes=tuple(("in0.shape[0]", "in0.shape[1]") for _ in outputs),
                      output_dtypes=tuple("in0" for _ in outputs), stages=tuple(stages))


def _local(n_in=2):
    return _rms_spec(kernel_id="local", input_names=tuple(f"in{i}" for i in range(n_in)))


def test_stage_plan_valid_and_walks_shapes():
    from metal_autotune_b200.autotuner_runtime.stages import shapes, wiring
    spec = _stage_spec([KernelStage(("in0", "in1"), ("tmp0",), _local()),
                        KernelStage(("tmp0", "in1"), ("out0",), _local())])
    plan, outs = wiring(spec)
    assert plan == [(0, 1), (2, 1)] and outs == (3,)
    _, out = shapes(spec, [(4, 16), (16,)], [torch.bfloat16, torch.bfloat16])
    assert out == [((4, 16), torch.bfloat16)]
    assert KernelSpec.from_json(spec.to_json()) == spec


@pytest.mark.parametrize("change,code", [("forward", "unbound"), ("overwrite", "rebind"), ("dead", "dead"),
                                         ("missing", "unproduced"), ("local_names", "local_inputs")])
def test_bad_stage_plans_rejected(change, code):
    from metal_autotune_b200.autotuner_runtime.stages import StageError, wiring
    s0 = KernelStage(("in0", "in1"), ("tmp0",), _local())
    s1 = KernelStage(("tmp0", "in1"), ("out0",), _local())
    if change == "forward":
        s0 = KernelStage(("tmp0", "in1"), ("tmp1",), _local())
    if change == "overwrite":
        s1 = KernelStage(("tmp0", "in1"), ("in0",), _local())
    if change == "dead":
        s1 = KernelStage(("in0", "in1"), ("out0",), _local())
    if change == "missing":
        s1 = KernelStage(("tmp0", "in1"), ("tmp1",), _local())
    if change == "local_names":
        s1 = KernelStage(("tmp0", "in1"), ("out0",), _rms_spec(kernel_id="x", input_names=("a", "b")))
    with pytest.raises(StageError) as e:
        wiring(_stage_spec([s0, s1]))
    assert e.value.code == code


# ------------------------------------------------------------ swap / apply
class Leaf(nn.Module):
    def __init__(self):
        super().__init__()
        self.w = nn.Parameter(torch.ones(3))

    def forward(self, x):
        return x * self.w


class Tree(nn.Module):
    def __init__(self):
        super().__init__()
        self.layers = nn.ModuleList([Leaf(), Leaf()])
        self.extra = {"a": Leaf()}


class Double(swap.ReplayWrapper):
    def forward(self, x):
        return 2 * self.wrapped(x)


def test_swap_install_uninstall_and_fallthrough():
    m = Tree()
    orig = swap.install(m, "layers.1", Double(m.layers[1]))
    assert isinstance(m.layers[1], Double)
    assert torch.equal(m.layers[1](torch.ones(3)), torch.full((3,), 2.0))
    assert m.layers[1].w is orig.w  # attribute falls through to the wrapped module
    assert any(p is orig.w for p in m.parameters())  # wrapped weights stay visible
    swap.uninstall(m, "layers.1", orig)
    assert m.layers[1] is orig
    with pytest.raises(KeyError, match="cannot resolve"):
        swap.resolve(m, "layers.7")
    with pytest.raises(ValueError):
        swap.resolve(m, "")


def test_state_signature_ignores_data():
    a = {"k": torch.zeros(2, 3), "n": 4}
    b = {"k": torch.ones(2, 3), "n": 4}
    assert swap.state_signature(a) == swap.state_signature(b)
    assert swap.state_signature(a) != swap.state_signature({"k": torch.zeros(3, 3), "n": 4})


def test_flatten_tensors_order():
    t = [torch.tensor(1), (torch.tensor(2), {"a": torch.tensor(3)}), 5]
    assert [int(x) for x in swap.flatten_tensors(t)] == [1, 2, 3]


def test_require_independent_models():
    a = Tree()
    swap.require_independent_models(a, Tree())
    b = Tree()
    b.layers[0] = a.layers[0]
    with pytest.raises(ValueError, match="reused a model module"):
        swap.require_independent_models(a, b)


def test_apply_bundle_installs_wrappers_on_tiny_qwen3():
    from pathlib import Path

    from metal_autotune_b200.autotuner_runtime.apply import apply
    from metal_autotune_b200.targets import qwen3
    model = qwen3.build(qwen3.TINY, device="cpu")
    bundle = Path(__file__).resolve().parents[1] / "metal_autotune_b200" / "bundles" / "qwen3_tiny"
    patched = apply(model, bundle)
    assert type(patched).__name__ == "W_qwen3_root"
    assert all(type(l).__name__ == "W_qwen3_layer" for l in patched.wrapped.layers)
    assert set(patched._specs) == {"quantized_embedding", "rms_norm", "lm_head", "logits_pick", "rms_norm_lm_head"}
    assert "rms_norm_qkv_qmm" in patched.wrapped.layers[0]._specs


# ------------------------------------------------------------ paired statistics
def test_paired_comparison_wins_and_losses():
    c = S.comparison_from_samples([10.0, 10.2, 9.9, 10.1], [8.0, 8.1, 7.9, 8.05])
    assert c.wins_by(0.5) and not c.loses_by(0.0)
    assert 0.75 < c.median_ratio < 0.85
    assert S.workload_win({"w": c})
    bad = S.comparison_from_samples([1.0, 1.0], [float("nan"), 1.0])
    assert not S.workload_win({"w": c, "v": bad})


def test_paired_means_needs_blocks():
    assert S.paired_means([1.0, 3.0, 2.0, 4.0]) == [2.0, 3.0]
    with pytest.raises(ValueError):
        S.paired_means([1.0, 2.0, 3.0])
    with pytest.raises(ValueError):
        S.comparison_from_samples([], [])
