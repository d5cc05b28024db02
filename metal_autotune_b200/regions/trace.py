"""The op stream of one model step, recorded at the aten level (the
reference's autotuner/trace/: recorder.py records MLX calls through patched
functions, types.py holds the Trace; here a TorchDispatchMode under
FakeTensorMode records every aten call, so nothing is computed and no device
memory is touched).

Each TraceNode is one call: its op (the aten overload), the arrays it reads
and writes (integer ids), their shapes and dtypes, its non-tensor arguments
with tensors replaced by ArrayRef(slot), and the module scope it ran in
(global forward hooks keep the stack of qualified module names). The Trace
also names the weights (id -> dotted path), the step's inputs and outputs,
each array's consumers, and the dead calls (outputs nobody reads).

replay(trace, lo, hi, bound) re-runs the recorded calls lo..hi on real
tensors (the region clock in price.py and the boundary checks use it,
trace/replay.py in the reference).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn
from torch.utils._python_dispatch import TorchDispatchMode
from torch.utils._pytree import tree_flatten, tree_map


@dataclass(frozen=True)
class ArrayRef:
    """A tensor argument's position in a node's in_arrays."""
    index: int


Spec = tuple  # (shape tuple, dtype name)


@dataclass
class TraceNode:
    seq: int
    op: str
    func: object                       # the OpOverload, for replay
    in_arrays: tuple
    out_arrays: tuple
    in_specs: tuple
    out_specs: tuple
    args: object                       # (args, kwargs) with tensors as ArrayRef
    module_stack: tuple                # enclosing module paths, outermost first ("" = root)

    @property
    def module_address(self) -> str:
        return self.module_stack[-1] if self.module_stack else ""


@dataclass
class Liveness:
    consumed_by: list = field(default_factory=list)


@dataclass
class Trace:
    workload: str
    nodes: list
    weights: dict                      # array id -> dotted path
    inputs: list                       # array ids of the step's tensor arguments
    step_outputs: list                 # array ids the step returns
    specs: dict                        # array id -> (shape, dtype)
    liveness: dict                     # array id -> Liveness
    dead: set                          # seqs whose outputs nobody reads

    def span_specs(self, lo: int, hi: int) -> dict:
        return self.specs


def _dtype_name(dt: torch.dtype) -> str:
    return str(dt).removeprefix("torch.")


class _Recorder(TorchDispatchMode):
    def __init__(self, ids, specs, stack):
        super().__init__()
        self.ids, self.specs, self.stack = ids, specs, stack
        self.nodes: list[TraceNode] = []
        self.keep: list = []  # holds recorded tensors so their id() stays unique

    def _id(self, t: torch.Tensor) -> int:
        k = id(t)
        aid = self.ids.get(k)
        if aid is None:
            aid = self.ids[k] = len(self.ids)
            self.specs[aid] = (tuple(t.shape), _dtype_name(t.dtype))
            self.keep.append(t)
        return aid

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        out = func(*args, **kwargs)
        if not any(isinstance(t, torch.Tensor) for t in tree_flatten(out)[0]):
            return out  # a metadata query (prim.device and the like): nothing computed
        ins: list[int] = []

        def ref(x):
            if isinstance(x, torch.Tensor):
                ins.append(self._id(x))
                return ArrayRef(len(ins) - 1)
            return x
        template = tree_map(ref, (args, kwargs))
        outs = [self._id(t) for t in tree_flatten(out)[0] if isinstance(t, torch.Tensor)]
        self.nodes.append(TraceNode(
            seq=len(self.nodes), op=str(func), func=func, in_arrays=tuple(ins), out_arrays=tuple(outs),
            in_specs=tuple(self.specs[a] for a in ins), out_specs=tuple(self.specs[a] for a in outs),
            args=template, module_stack=tuple(self.stack)))
        return out


def record(module: nn.Module, args: tuple, workload: str = "step") -> Trace:
    """The aten op stream of module(*args), on fake tensors of the same shapes."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    names = {id(m): n for n, m in module.named_modules(remove_duplicate=False)}
    weights = {}
    for prefix, sub in module.named_modules(remove_duplicate=False):
        for attr, t in list(sub._parameters.items()) + list(sub._buffers.items()):
            if t is not None:
                weights.setdefault(f"{prefix}.{attr}" if prefix else attr, t)
    stack: list[str] = []

    def pre(mod, _inp):
        stack.append(names.get(id(mod), type(mod).__name__))

    def post(mod, _inp, _out):
        if stack:
            stack.pop()
    h1 = nn.modules.module.register_module_forward_pre_hook(pre)
    h2 = nn.modules.module.register_module_forward_hook(post)
    ids: dict[int, int] = {}
    specs: dict[int, tuple] = {}
    try:
        with FakeTensorMode(allow_non_fake_inputs=False) as fm:
            fw = {k: fm.from_tensor(v) for k, v in weights.items()}
            fa = tuple(fm.from_tensor(a) if isinstance(a, torch.Tensor) else a for a in args)
            rec = _Recorder(ids, specs, stack)
            weight_ids = {rec._id(t): k for k, t in fw.items()}
            input_ids = [rec._id(a) for a in fa if isinstance(a, torch.Tensor)]
            with rec:
                out = torch.func.functional_call(module, fw, fa)
            outputs = [rec._id(t) for t in tree_flatten(out)[0] if isinstance(t, torch.Tensor)]
    finally:
        h1.remove()
        h2.remove()
    nodes = rec.nodes
    live = {aid: Liveness() for aid in specs}
    for n in nodes:
        for a in n.in_arrays:
            live[a].consumed_by.append(n.seq)
    outs = set(outputs)
    dead = {n.seq for n in nodes if n.out_arrays and all(not live[a].consumed_by and a not in outs
                                                         for a in n.out_arrays)}
    return Trace(workload, nodes, weight_ids, input_ids, outputs, specs, live, dead)


def _restore(template, arrays):
    return tree_map(lambda x: arrays[x.index] if isinstance(x, ArrayRef) else x, template,
                    is_leaf=lambda x: isinstance(x, ArrayRef))


def replay(trace: Trace, lo: int, hi: int, bound: dict) -> dict:
    """Run the recorded calls lo..hi (inclusive) with `bound` (array id ->
    tensor) supplying every array they read from outside; returns bound
    extended with every array they produce."""
    env = dict(bound)
    for node in trace.nodes[lo:hi + 1]:
        args, kwargs = _restore(node.args, [env[a] for a in node.in_arrays])
        out = node.func(*args, **kwargs)
        flat = [t for t in tree_flatten(out)[0] if isinstance(t, torch.Tensor)]
        for aid, t in zip(node.out_arrays, flat):
            env[aid] = t
    return env
