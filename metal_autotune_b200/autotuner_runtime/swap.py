"""Module swap on torch.nn.Module trees (the reference's
autotuner_runtime/swap.py:17-152, which does this on mlx.nn trees).

Scope addresses are dot paths ("layers.3.mlp"); the swap itself is parent
attribute assignment, or index assignment for children held in lists /
ModuleLists / dicts. A ReplayWrapper keeps the wrapped module as a child, so
parameters() and named_modules() still see the original weights, and
unknown attributes fall through to the wrapped module.
"""
from __future__ import annotations

import torch
import torch.nn as nn


def flatten_tensors(tree: object) -> list[torch.Tensor]:
    """Every tensor of a nested list/tuple/dict tree, depth-first in order
    (swap.py:20-38), walked with an explicit stack."""
    out: list[torch.Tensor] = []
    stack = [tree]
    while stack:
        obj = stack.pop()
        if isinstance(obj, torch.Tensor):
            out.append(obj)
        elif isinstance(obj, (list, tuple)):
            stack.extend(reversed(obj))
        elif isinstance(obj, dict):
            stack.extend(reversed(list(obj.values())))
    return out


flatten_arrays = flatten_tensors  # the reference's name


def state_signature(value):
    """Structure, scalars and tensor shapes/dtypes of state, never tensor data
    (swap.py:40-64): guards replays whose Python branches depended on state."""
    seen: dict[int, int] = {}

    def visit(obj):
        if isinstance(obj, torch.Tensor):
            return ("tensor", tuple(obj.shape), str(obj.dtype).removeprefix("torch."))
        if obj is None or isinstance(obj, (str, int, float, bool)):
            return obj
        if id(obj) in seen:
            return ("alias", seen[id(obj)])
        seen[id(obj)] = len(seen)
        if isinstance(obj, dict):
            return ("dict", tuple((k, visit(v)) for k, v in sorted(obj.items())))
        if isinstance(obj, (tuple, list)):
            return (type(obj).__name__, tuple(visit(v) for v in obj))
        if hasattr(obj, "__dict__"):
            return (type(obj).__name__, visit(vars(obj)))
        raise TypeError(f"cannot describe state field of type {type(obj).__name__}")

    return visit(value)


class ReplayWrapper(nn.Module):
    """Base of region wrappers: subclasses implement forward() as the scope's
    op sequence with region kernels spliced in (swap.py:67-81)."""

    def __init__(self, wrapped: nn.Module, specs: dict | None = None):
        super().__init__()
        self.wrapped = wrapped
        object.__setattr__(self, "_specs", dict(specs or {}))

    def __getattr__(self, name):
        try:
            return super().__getattr__(name)
        except AttributeError:
            if name == "wrapped" or "wrapped" not in self._modules:
                raise
            return getattr(self._modules["wrapped"], name)


def require_independent_models(first, second):
    """Weights may be shared; mutable modules must belong to one arm (swap.py:84-95)."""
    if not isinstance(first, nn.Module) or not isinstance(second, nn.Module):
        return
    originals = {id(m) for m in first.modules()}
    for path, m in second.named_modules():
        if id(m) in originals:
            raise ValueError(f"build() reused a model module at {path or '<root>'}; return fresh model "
                             "and layer instances on every call. Weight tensors may be shared.")


def _child(obj: object, key: str, full_path: str):
    try:
        if isinstance(obj, (list, tuple, nn.ModuleList, nn.Sequential)):
            return obj[int(key)]
        if isinstance(obj, (dict, nn.ModuleDict)):
            return obj[key]
        return getattr(obj, key)
    except (AttributeError, KeyError, IndexError, ValueError, TypeError) as e:
        raise KeyError(f"cannot resolve scope address {full_path!r}: no child {key!r} on "
                       f"{type(obj).__name__} ({e}); the model tree changed since the trace") from None


def resolve(model: object, path: str):
    """path -> (parent, key, child); the root has no parent (swap.py:98-109)."""
    if path == "":
        raise ValueError("the root scope has no parent to swap under")
    parts = path.split(".")
    obj = model
    for p in parts[:-1]:
        obj = _child(obj, p, path)
    return obj, parts[-1], _child(obj, parts[-1], path)


def resolve_value(model: object, path: str):
    """Weights and state by dot path through modules, dicts and sequences."""
    obj = model
    for p in path.split(".") if path else []:
        obj = _child(obj, p, path)
    return obj


def _assign(parent: object, key: str, value: object) -> None:
    if isinstance(parent, (list, nn.ModuleList, nn.Sequential)):
        parent[int(key)] = value
    elif isinstance(parent, nn.ModuleDict) or (isinstance(parent, dict) and not isinstance(parent, nn.Module)):
        parent[key] = value
    elif isinstance(parent, tuple):
        raise TypeError("cannot swap a child living in a tuple; the model must use lists")
    else:
        setattr(parent, key, value)


def install(model: object, path: str, wrapper: nn.Module) -> object:
    """Swap `wrapper` in at `path`; returns the previous occupant for rollback."""
    parent, key, occupant = resolve(model, path)
    _assign(parent, key, wrapper)
    return occupant


def uninstall(model: object, path: str, occupant: object) -> None:
    parent, key, _ = resolve(model, path)
    _assign(parent, key, occupant)
