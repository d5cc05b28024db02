"""Installing region wrappers into torch.nn.Module trees (the reference does
this on mlx.nn trees: autotuner_runtime/swap.py:17-152).

A scope address is a dot path of child keys from the model's root
("layers.3.mlp"). A key names an attribute, an index into a list-like
container (ModuleList, Sequential, list, tuple) or a key of a dict-like one
(ModuleDict, dict). `Scope` parses an address once and walks it with one
reader and one writer per container kind; `install` puts a wrapper at an
address and returns what it displaced, `uninstall` puts that back.

A ReplayWrapper keeps the module it wraps as its child `wrapped`, so the
model's parameters and module names still reach the original weights, and
an attribute the wrapper does not have is read from the wrapped module.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator

import torch
import torch.nn as nn

_LISTLIKE = (list, tuple, nn.ModuleList, nn.Sequential)
_DICTLIKE = (dict, nn.ModuleDict)


def _read(node: object, key: str) -> object:
    if isinstance(node, _LISTLIKE):
        return node[int(key)]
    if isinstance(node, _DICTLIKE):
        return node[key]
    return getattr(node, key)


def _write(node: object, key: str, value: object) -> None:
    if isinstance(node, tuple):
        raise TypeError("a child held in a tuple cannot be replaced; the model must keep it in a list")
    if isinstance(node, _LISTLIKE):
        node[int(key)] = value
    elif isinstance(node, nn.ModuleDict) or (isinstance(node, dict) and not isinstance(node, nn.Module)):
        node[key] = value
    else:
        setattr(node, key, value)


@dataclass(frozen=True)
class Scope:
    """A parsed scope address."""
    path: str

    @property
    def keys(self) -> tuple[str, ...]:
        return tuple(self.path.split(".")) if self.path else ()

    def _step(self, node: object, key: str) -> object:
        try:
            return _read(node, key)
        except (AttributeError, KeyError, IndexError, ValueError, TypeError) as e:
            raise KeyError(f"cannot resolve scope address {self.path!r}: {type(node).__name__} has no child "
                           f"{key!r} ({e}); the model tree changed since the bundle was recorded") from None

    def walk(self, root: object) -> Iterator[object]:
        """The nodes along the address, root excluded, outermost first."""
        node = root
        for key in self.keys:
            node = self._step(node, key)
            yield node

    def get(self, root: object) -> object:
        node = root
        for node in self.walk(root):
            pass
        return node

    def parent(self, root: object) -> tuple[object, str]:
        if not self.keys:
            raise ValueError("the root scope has no parent to install a wrapper under")
        head = Scope(".".join(self.keys[:-1]))
        return head.get(root), self.keys[-1]


def resolve(model: object, path: str) -> tuple[object, str, object]:
    """(parent, key, child) at an address (swap.py:98-109); the root has none."""
    scope = Scope(path)
    parent, key = scope.parent(model)
    return parent, key, scope._step(parent, key)


def resolve_value(model: object, path: str) -> object:
    """A weight, a state field or a module by address ("" is the model)."""
    return Scope(path).get(model)


def install(model: object, path: str, wrapper: nn.Module) -> object:
    """Put `wrapper` at `path`; returns the displaced occupant for uninstall."""
    parent, key, occupant = resolve(model, path)
    _write(parent, key, wrapper)
    return occupant


def uninstall(model: object, path: str, occupant: object) -> None:
    parent, key = Scope(path).parent(model)
    _write(parent, key, occupant)


class ReplayWrapper(nn.Module):
    """Base of region wrappers (swap.py:67-81): a subclass's forward runs the
    scope's op sequence with region kernels in place of their ops; `_specs`
    holds the kernel specs by id."""

    def __init__(self, wrapped: nn.Module, specs: dict | None = None):
        super().__init__()
        self.wrapped = wrapped
        object.__setattr__(self, "_specs", dict(specs or {}))

    def __getattr__(self, name):
        try:
            return super().__getattr__(name)
        except AttributeError:
            inner = self._modules.get("wrapped")
            if name == "wrapped" or inner is None:
                raise
            return getattr(inner, name)


def require_independent_models(first: object, second: object) -> None:
    """Two builds compared side by side may share weight tensors but not
    modules: installing wrappers into one must not change the other
    (swap.py:84-95)."""
    if not (isinstance(first, nn.Module) and isinstance(second, nn.Module)):
        return
    mine = {id(m) for m in first.modules()}
    shared = next((path for path, m in second.named_modules() if id(m) in mine), None)
    if shared is not None:
        raise ValueError(f"build() reused a model module at {shared or '<root>'}; return fresh model and layer "
                         "instances on every call. Weight tensors may be shared.")


def flatten_tensors(tree: object) -> list[torch.Tensor]:
    """The tensors of a nested list / tuple / dict, depth-first in order
    (swap.py:20-38)."""
    def leaves(node):
        if isinstance(node, torch.Tensor):
            yield node
        elif isinstance(node, (list, tuple)):
            for child in node:
                yield from leaves(child)
        elif isinstance(node, dict):
            for child in node.values():
                yield from leaves(child)
    return list(leaves(tree))


def state_signature(value: object) -> object:
    """What a replay's Python branches may have depended on (swap.py:40-64):
    the structure of a state object, its scalars, and its tensors' shapes and
    dtypes, never tensor contents. An object met twice is named by the
    order it was first met, so aliasing is part of the signature."""
    order: dict[int, int] = {}

    def describe(node):
        if isinstance(node, torch.Tensor):
            return ("tensor", tuple(node.shape), str(node.dtype).removeprefix("torch."))
        if node is None or isinstance(node, (str, int, float, bool)):
            return node
        if id(node) in order:
            return ("alias", order[id(node)])
        order[id(node)] = len(order)
        if isinstance(node, dict):
            return ("dict", tuple((k, describe(node[k])) for k in sorted(node)))
        if isinstance(node, (list, tuple)):
            return (type(node).__name__, tuple(describe(v) for v in node))
        if hasattr(node, "__dict__"):
            return (type(node).__name__, describe(vars(node)))
        raise TypeError(f"cannot describe state field of type {type(node).__name__}")

    return describe(value)
