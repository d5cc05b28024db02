"""apply(): install a region bundle onto a freshly built model
(the reference's autotuner_runtime/apply.py:19-67).

A bundle directory holds
  swap_table.json      [{"scope_path": "layers.0", "wrapper_class": "...", "kernel_ids": [...]}, ...]
  patch/wrappers.py    the wrapper classes (ReplayWrapper subclasses)
  kernels/*.launch.json  one KernelSpec per kernel id (cuda records)
An entry at the root scope ("") wraps the model itself, so callers use the
return value. Works in a fresh process.
"""
from __future__ import annotations

import importlib.util
import json
from pathlib import Path

from . import kernels as _kernels
from .swap import install, resolve


def load_specs(bundle_dir: str | Path) -> dict[str, _kernels.KernelSpec]:
    specs = {}
    for p in sorted((Path(bundle_dir) / "kernels").glob("*.launch.json")):
        spec = _kernels.load_spec(p)
        specs[spec.kernel_id] = spec
    return specs


def load_wrappers(bundle_dir: str | Path, prefix: str = ""):
    path = Path(bundle_dir) / "patch" / f"{prefix}wrappers.py"
    mod_spec = importlib.util.spec_from_file_location(f"mt_bundle_wrappers_{abs(hash(str(path)))}", path)
    module = importlib.util.module_from_spec(mod_spec)
    mod_spec.loader.exec_module(module)
    return module


def apply(model: object, bundle_dir: str | Path, *, baseline: bool = False) -> object:
    bundle_dir = Path(bundle_dir)
    prefix = "baseline_" if baseline else ""
    table = json.loads((bundle_dir / f"{prefix}swap_table.json").read_text())
    wrappers = load_wrappers(bundle_dir, prefix)
    specs = {} if baseline else load_specs(bundle_dir)
    patched = model
    for entry in table:
        cls = getattr(wrappers, entry["wrapper_class"])
        try:
            kspecs = {kid: specs[kid] for kid in entry["kernel_ids"]}
        except KeyError as e:
            raise KeyError(f"swap table names kernel {e} that the bundle does not ship") from None
        path = entry["scope_path"]
        if path == "":
            patched = cls(patched, kspecs)
        else:
            _, _, original = resolve(patched, path)
            install(patched, path, cls(original, kspecs))
    return patched
