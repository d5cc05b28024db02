"""Portable definitions of custom CUDA region kernels (the reference's
autotuner_runtime/captured_kernels.py:1-86, which records
mx.fast.metal_kernel definitions).

A definition here is the JSON of a `cuda` record (entry-point symbol and
argument bindings) plus output shapes/dtypes: enough to rebuild a
LoadedKernel in a fresh process. `capture` wraps a factory so the definition
travels with the kernel object; `captured(key)` rebuilds one definition at
most once; an optional recorder sees every call.
"""
from __future__ import annotations

import json
from contextlib import contextmanager
from functools import lru_cache

from . import kernels as _kernels

_recorder = None


def activate(recorder) -> None:
    global _recorder
    if _recorder is not None:
        raise RuntimeError("a kernel recorder is already active")
    _recorder = recorder


def deactivate(recorder) -> None:
    global _recorder
    if _recorder is recorder:
        _recorder = None


def definition_key(definition: dict) -> str:
    return json.dumps(definition, sort_keys=True, separators=(",", ":"), allow_nan=False)


class CapturedKernel:
    """A LoadedKernel that remembers the definition it was built from."""

    def __init__(self, kernel: _kernels.LoadedKernel, definition: dict):
        self._kernel = kernel
        self.definition = definition

    def __call__(self, inputs, **kwargs):
        out = self._kernel(inputs, **kwargs)
        rec = _recorder
        if rec is not None and getattr(rec, "recording", False):
            rec.record_kernel(self.definition, inputs, out)
        return out


def _build(kwargs: dict) -> _kernels.LoadedKernel:
    spec = _kernels.KernelSpec(
        kernel_id=kwargs.get("name", kwargs["cuda"]["symbol"]), name=kwargs.get("name", kwargs["cuda"]["symbol"]),
        input_names=tuple(kwargs["input_names"]), output_names=tuple(kwargs["output_names"]),
        cuda=kwargs["cuda"], output_shapes=tuple(tuple(s) for s in kwargs["output_shapes"]),
        output_dtypes=tuple(kwargs["output_dtypes"]))
    return _kernels.LoadedKernel(spec)


def capture(**kwargs) -> CapturedKernel:
    """Build a kernel from keyword arguments (name, input_names, output_names,
    cuda, output_shapes, output_dtypes) and keep the definition."""
    kernel = _build(kwargs)
    definition = json.loads(definition_key({"version": 1, "kwargs": kwargs}))
    return CapturedKernel(kernel, definition)


@lru_cache(maxsize=256)
def captured(key: str) -> CapturedKernel:
    """Rebuild a kernel from its definition key, once per definition."""
    definition = json.loads(key)
    if definition.get("version") != 1:
        raise ValueError("unsupported captured kernel definition version")
    return CapturedKernel(_build(definition["kwargs"]), definition)


@contextmanager
def capture_construction():
    """Scope in which kernels built through `capture` are recorded by an active
    recorder; a no-op scope otherwise (kept for the reference's API shape)."""
    yield
