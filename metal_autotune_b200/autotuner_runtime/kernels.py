"""Kernel specs and the one call site of the region contract, on libmt.so.

Mirrors the reference's autotuner_runtime/kernels.py:34-268. A KernelSpec is
the serialisable description of a region kernel: input/output names, output
shapes and dtypes in the launch grammar, a fallback predicate, the accepted
input signatures, optional multi-stage dataflow. Where the reference holds a
Metal body and header for mx.fast.metal_kernel, a spec here holds a `cuda`
record binding the region to one libmt.so entry point:

    "cuda": {"symbol": "mt_quantized_matmul",
             "args": [{"in": 0}, {"in": 1}, ..., {"out": 0},
                      {"expr": "in0.shape[0] * in0.shape[1]"},  # int64 from the grammar
                      {"int": 64}, {"float": 1e-6}, {"dtype": "in0"},
                      {"stride": [0, 1]},                         # input 0, axis 1
                      {"null": true},
                      {"scalar": "offset"},                       # runtime value from `scalars=`
                      {"workspace": {"query": "mt_qmm_workspace_bytes",
                                     "args": [{"expr": ...}, {"int": 4}, ...]}},
                      {"stream": true}]}

The entry points own their launch geometry, so `grid`/`threadgroup` are kept
only for format compatibility. Outputs are allocated by torch from
`output_shapes`/`output_dtypes`; `init_value` poisons them before the launch
(the harness owns it, kernels.py:1-9). The launch — fallback decision,
output shapes, resolved integer arguments — is evaluated once per call
signature (shapes, dtypes) and cached (kernels.py:102-188). Like the
reference, the kernel cache is a module global: one thread, one stream.
"""
from __future__ import annotations

import ctypes as C
import importlib
import json
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import NamedTuple

import torch

from .. import lib as _mt
from .grammar import Expr

DTYPES = {
    "bool": torch.bool, "uint8": torch.uint8, "uint16": torch.uint16, "uint32": torch.uint32,
    "uint64": torch.uint64, "int8": torch.int8, "int16": torch.int16, "int32": torch.int32,
    "int64": torch.int64, "float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
}
DTYPE_NAMES = {v: k for k, v in DTYPES.items()}


def dtype_name(dt: torch.dtype) -> str:
    return DTYPE_NAMES[dt]


@dataclass(frozen=True)
class KernelSpec:
    kernel_id: str
    name: str                                   # a valid C identifier
    input_names: tuple[str, ...]
    output_names: tuple[str, ...]
    cuda: dict | None = None                    # {"symbol": ..., "args": [...]}; None for staged specs
    grid: tuple[str, str, str] = ("1", "1", "1")          # informational: entry points own geometry
    threadgroup: tuple[str, str, str] = ("1", "1", "1")
    output_shapes: tuple[tuple[str, ...], ...] = ()       # one expr tuple per output
    output_dtypes: tuple[str, ...] = ()                   # dtype names or "inK"
    fallback_predicate: str | None = None                 # true -> the original ops take the call
    ensure_row_contiguous: bool = True
    input_signature: list | None = None                   # exact [[shape], dtype] per input
    input_signatures: list | None = None                  # allowed alternatives
    stages: tuple["KernelStage", ...] = ()
    reassociates: bool = False  # adds in its own order: checked within tolerance, never bitwise

    def to_json(self) -> str:
        d = {k: getattr(self, k) for k in self.__dataclass_fields__}
        d["stages"] = [{"inputs": list(s.inputs), "outputs": list(s.outputs), "kernel": json.loads(s.kernel.to_json())}
                       for s in self.stages]
        return json.dumps(d, indent=1)

    @staticmethod
    def from_json(text: str) -> "KernelSpec":
        d = json.loads(text)
        for k in ("input_names", "output_names", "grid", "threadgroup", "output_dtypes"):
            if k in d:
                d[k] = tuple(d[k])
        d["output_shapes"] = tuple(tuple(s) for s in d.get("output_shapes", ()))
        d["stages"] = tuple(KernelStage(tuple(s["inputs"]), tuple(s["outputs"]),
                                        KernelSpec.from_json(json.dumps(s["kernel"])))
                            for s in d.get("stages", ()))
        return KernelSpec(**d)

    def __hash__(self) -> int:
        return hash(self.kernel_id)


@dataclass(frozen=True)
class KernelStage:
    inputs: tuple[str, ...]   # outer inN or an earlier tmpN/outN
    outputs: tuple[str, ...]  # new tmpN/outN names
    kernel: KernelSpec        # local ABI: in0.. and out0..


def load_spec(path: str | Path) -> KernelSpec:
    """Rebuild a spec from <id>.launch.json."""
    return KernelSpec.from_json(Path(path).read_text())


def write_spec(directory: str | Path, spec: KernelSpec) -> Path:
    p = Path(directory) / f"{spec.kernel_id}.launch.json"
    p.write_text(spec.to_json() + "\n")
    return p


class Launch(NamedTuple):
    """One call signature's resolved launch, or the fact that the fallback covers it."""
    fallback: bool
    output_shapes: list | None = None
    output_dtypes: list | None = None
    args: list | None = None   # per ABI argument: ("in", i) / ("out", i) / ("val", ctypes value) / ...


LAUNCH_CACHE_MAX = 64


def _resolve_dtype(name: str, dtypes: list[torch.dtype]) -> torch.dtype:
    if name.startswith("in") and name[2:].isdigit():
        return dtypes[int(name[2:])]
    return DTYPES[name]


class LoadedKernel:
    """A spec bound to its libmt.so entry point plus parsed launch expressions."""

    def __init__(self, spec: KernelSpec):
        self.spec = spec
        self._stages = None
        if spec.stages:
            from .stages import build_graph
            self._graph = build_graph(spec)
            self._stage_outputs = self._graph.outputs
            self._stages = [(LoadedKernel(node.kernel), node.reads) for node in self._graph.nodes]
        elif spec.cuda is None:
            raise ValueError(f"kernel {spec.kernel_id}: a spec needs a cuda record or stages")
        self._fn = None
        if spec.cuda is not None:
            sym = spec.cuda["symbol"]
            if sym not in _mt.SIGNATURES:
                raise ValueError(f"kernel {spec.kernel_id}: {sym} is not a libmt entry point")
            self._fn = getattr(_mt.load(), sym)
            self._symbol = sym
            self._arg_exprs = [self._parse_arg(a) for a in spec.cuda["args"]]
        self._out_shapes = tuple(tuple(Expr(e) for e in s) for s in spec.output_shapes)
        self._fallback = Expr(spec.fallback_predicate) if spec.fallback_predicate else None
        self._launches: dict[tuple, Launch] = {}

    @staticmethod
    def _parse_arg(a: dict):
        if "expr" in a:
            return ("expr", Expr(a["expr"]))
        if "workspace" in a:
            w = a["workspace"]
            return ("workspace", w["query"], [LoadedKernel._parse_arg(x) for x in w.get("args", [])])
        return ("raw", a)

    def _eval_scalar(self, parsed, shapes, dtypes):
        kind = parsed[0]
        if kind == "expr":
            return int(parsed[1].evaluate(shapes))
        a = parsed[1]
        if "int" in a:
            return int(a["int"])
        if "float" in a:
            return float(a["float"])
        if "dtype" in a:
            return _mt.dtype_code(_resolve_dtype(a["dtype"], dtypes))
        raise ValueError(f"argument {a} is not a scalar")

    def launch(self, inputs: list[torch.Tensor], checked_elsewhere: bool = False) -> Launch:
        """checked_elsewhere: the caller serves only sizes it checked this kernel
        at, so the recorded signatures do not bound the call; the fallback
        predicate still does (kernels.py:137-141)."""
        key = (checked_elsewhere, *((tuple(a.shape), a.dtype) for a in inputs))
        launch = self._launches.get(key)
        if launch is not None:
            return launch
        shapes = [s for s, _ in key[1:]]
        dtypes = [d for _, d in key[1:]]
        sig = [[list(s), dtype_name(d)] for s, d in zip(shapes, dtypes)]
        spec = self.spec
        if ((not checked_elsewhere and (
                (spec.input_signature is not None and sig != spec.input_signature)
                or (spec.input_signatures is not None and sig not in spec.input_signatures)))
                or (self._fallback is not None and self._fallback.evaluate(shapes))):
            launch = Launch(fallback=True)
        else:
            out_shapes = [tuple(int(e.evaluate(shapes)) for e in s) for s in self._out_shapes]
            out_dtypes = [_resolve_dtype(d, dtypes) for d in spec.output_dtypes]
            args = None
            if self._stages is not None:
                _, outs = self._graph.walk_shapes(shapes, dtypes)
                if [(tuple(s), d) for s, d in outs] != list(zip(out_shapes, out_dtypes)):
                    raise ValueError("stage results do not match the region's output shapes/dtypes")
            else:
                args = []
                for parsed in self._arg_exprs:
                    kind = parsed[0]
                    if kind == "workspace":
                        q = getattr(_mt.load(), parsed[1])
                        nbytes = int(q(*[self._eval_scalar(x, shapes, dtypes) for x in parsed[2]]))
                        args.append(("workspace", nbytes))
                        continue
                    if kind == "expr":
                        args.append(("val", int(parsed[1].evaluate(shapes))))
                        continue
                    a = parsed[1]
                    if "in" in a:
                        args.append(("in", int(a["in"])))
                    elif "out" in a:
                        args.append(("out", int(a["out"])))
                    elif "stride" in a:
                        args.append(("stride", tuple(a["stride"])))
                    elif "null" in a:
                        args.append(("val", None))
                    elif "scalar" in a:
                        args.append(("scalar", a["scalar"]))
                    elif "stream" in a:
                        args.append(("stream", None))
                    else:
                        args.append(("val", self._eval_scalar(parsed, shapes, dtypes)))
            launch = Launch(False, out_shapes, out_dtypes, args)
        if len(self._launches) >= LAUNCH_CACHE_MAX:
            self._launches.clear()
        self._launches[key] = launch
        return launch

    def fallback_fires(self, inputs: list[torch.Tensor]) -> bool:
        return self.launch(inputs).fallback

    def __call__(self, inputs: list[torch.Tensor], init_value: float | None = None,
                 launch: Launch | None = None, outputs: list[torch.Tensor] | None = None,
                 scalars: dict | None = None) -> list[torch.Tensor]:
        launch = launch or self.launch(inputs)
        if launch.fallback:
            raise ValueError(f"kernel {self.spec.kernel_id}: these shapes are the fallback's; "
                             "the original ops take them")
        if self.spec.ensure_row_contiguous:
            inputs = [a if a.is_contiguous() else a.contiguous() for a in inputs]
        if self._stages is not None:
            buffers = list(inputs)
            for kernel, idx in self._stages:
                buffers.extend(kernel([buffers[i] for i in idx], init_value=init_value, scalars=scalars))
            return [buffers[i] for i in self._stage_outputs]
        dev = inputs[0].device if inputs else torch.device("cuda", torch.cuda.current_device())
        if outputs is None:
            outputs = [torch.empty(s, dtype=d, device=dev) for s, d in zip(launch.output_shapes, launch.output_dtypes)]
        if init_value is not None:
            for o in outputs:
                o.fill_(init_value)
        cargs = []
        for kind, v in launch.args:
            if kind == "in":
                cargs.append(_mt._ptr(inputs[v]))
            elif kind == "out":
                cargs.append(_mt._ptr(outputs[v]))
            elif kind == "val":
                cargs.append(v)
            elif kind == "stride":
                cargs.append(inputs[v[0]].stride(v[1]))
            elif kind == "stream":
                cargs.append(_mt._stream())
            elif kind == "scalar":
                if scalars is None or v not in scalars:
                    raise ValueError(f"kernel {self.spec.kernel_id}: runtime scalar {v!r} not supplied")
                cargs.append(scalars[v])
            elif kind == "workspace":
                ws = _mt.Workspace.get(v, dev.index)
                cargs.append(ws.ptr)
                cargs.append(ws.nbytes)
        rc = self._fn(*cargs)
        _mt.CALLS[0] += 1
        if rc != 0:
            _mt._check(rc, self._symbol)
        return outputs


def imported(path: str):
    """The model's own function by import path (a wrapper calls it where the
    recording saw a compiled section, kernels.py:223-227)."""
    module, _, name = path.rpartition(".")
    return getattr(importlib.import_module(module), name)


_cache: dict[str, LoadedKernel] = {}


def _loaded(spec: KernelSpec) -> LoadedKernel:
    lk = _cache.get(spec.kernel_id)
    if lk is None or lk.spec is not spec:
        lk = LoadedKernel(spec)
        _cache[spec.kernel_id] = lk
    return lk


def fallback_fires(spec: KernelSpec, inputs: list[torch.Tensor]) -> bool:
    """True when these shapes are not covered and the wrapper must run the original ops."""
    return _loaded(spec).fallback_fires(inputs)


def call(spec: KernelSpec, inputs: list[torch.Tensor], init_value: float | None = None,
         launch: Launch | None = None, outputs: list[torch.Tensor] | None = None,
         scalars: dict | None = None) -> list[torch.Tensor]:
    """The replacement call site (kernels.py:247-251). `outputs` lets a caller
    supply the output buffers; `scalars` carries runtime values such as a
    cache offset, which the reference records as literals guarded by the
    state signature (tests/test_rope_offset.py)."""
    return _loaded(spec)(inputs, init_value=init_value, launch=launch, outputs=outputs, scalars=scalars)


def try_call(spec: KernelSpec, inputs: list[torch.Tensor], outputs: list[torch.Tensor] | None = None,
             scalars: dict | None = None) -> list[torch.Tensor] | None:
    """What a wrapper calls: the outputs, or None when the fallback covers
    these shapes and the wrapper runs the original ops (kernels.py:254-259)."""
    lk = _loaded(spec)
    launch = lk.launch(inputs)
    return None if launch.fallback else lk(inputs, launch=launch, outputs=outputs, scalars=scalars)


def try_sized(spec: KernelSpec, inputs: list[torch.Tensor], init_value: float | None = None,
              outputs: list[torch.Tensor] | None = None, scalars: dict | None = None) -> list[torch.Tensor] | None:
    """try_call for a size-generic wrapper: recorded signatures do not bound the
    call, the fallback predicate still does (kernels.py:262-268)."""
    lk = _loaded(spec)
    launch = lk.launch(inputs, checked_elsewhere=True)
    return None if launch.fallback else lk(inputs, init_value=init_value, launch=launch, outputs=outputs,
                                           scalars=scalars)
