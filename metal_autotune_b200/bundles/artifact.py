"""Fresh-process check and timing of a region bundle (the reference's
exported-artifact tools, autotuner/artifact/validate.py:179-230 and
autotuner/artifact/benchmark.py; docs/artifacts.md:174-190).

A bundle directory describes how to rebuild its target and what to run it
on (bundle.json):

  "builder":  "package.module:function"  builds the unpatched target
  "config":   name of a config object in the builder's module (or null)
  "seed":     the builder's seed
  "entry":    how one workload is run and which outputs are compared
              (a key of ENTRIES below)
  "workloads": {label: {"file": "workloads/<label>.safetensors"} or
                       {"seeded": {"kind": "randn" | "randint", "shape": [...],
                                   "dtype": "...", "seed": s, "high": n}}}
  "correctness_rule": "baseline_tolerance" | "exact"
  "tolerances": {"rtol": r, "atol": a} (optional; else per-dtype defaults)
  "final_benchmark": {"pairs": 4, "warmup_steps": 3, "steps": 5}

`validate` builds the original model and, separately, a second copy with the
bundle applied (apply() installs wrappers in place, so the two cannot share
one module tree), then for every workload runs each model twice: both must
repeat bit for bit, and every patched output must equal the original's
under the recorded rule (numeric.check: the GPU output-diff reduction).
`benchmark` runs validate first, then times whole sequences of consecutive
steps of both models, alternated in both orders (sequence.compare_sequences
on CUDA events). Both run in a fresh process:

  python -m metal_autotune_b200.bundles.validate  <bundle_dir> [--json out]
  python -m metal_autotune_b200.bundles.benchmark <bundle_dir> [--json out]
"""
from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

import torch

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32, "int32": torch.int32}


# ------------------------------------------------------------------ entries
def _qwen3_prefill(model, inputs, state):
    """One prefill of the prompt from an empty KV cache: the last position's logits."""
    from ..targets import qwen3
    (tokens,) = inputs
    if "cache" not in state:
        state["cache"] = qwen3.KVCache(model.cfg, device="cuda")
    cache = state["cache"]
    cache.reset()
    model(tokens, cache)
    return [model.last_logits]


def _whisper_encoder(model, inputs, state):
    (mel,) = inputs
    return [model(mel)]


def _mamba_prefill(model, inputs, state):
    (tokens,) = inputs
    return [model(tokens)[1]]


def _tiny_mlp(model, inputs, state):
    (x,) = inputs
    return [model(x)]


ENTRIES = {"qwen3_prefill": _qwen3_prefill, "whisper_encoder": _whisper_encoder, "mamba_prefill": _mamba_prefill,
           "tiny_mlp": _tiny_mlp}


# ------------------------------------------------------------------ loading
def read_meta(bundle_dir: Path) -> dict:
    return json.loads((Path(bundle_dir) / "bundle.json").read_text())


def build_target(meta: dict, device="cuda"):
    mod_name, _, fn_name = meta["builder"].partition(":")
    mod = importlib.import_module(mod_name)
    kwargs = {"device": device}
    if meta.get("seed") is not None:
        kwargs["seed"] = meta["seed"]
    args = (getattr(mod, meta["config"]),) if meta.get("config") else ()
    out = getattr(mod, fn_name)(*args, **kwargs)
    return out[0] if isinstance(out, tuple) else out  # builders that also return an input keep only the model


def workload_inputs(bundle_dir: Path, entry: dict, device="cuda") -> list[torch.Tensor]:
    if "file" in entry:
        from safetensors.torch import load_file
        data = load_file(str(Path(bundle_dir) / entry["file"]))
        return [data[f"i{k}"].to(device) for k in range(len(data))]
    spec = entry["seeded"]
    g = torch.Generator().manual_seed(spec["seed"])
    shape = tuple(spec["shape"])
    if spec["kind"] == "randint":
        t = torch.randint(0, spec["high"], shape, generator=g, dtype=torch.int64).to(DTYPES[spec["dtype"]])
    else:
        t = torch.randn(shape, generator=g, dtype=torch.float32).to(DTYPES[spec["dtype"]])
    return [t.to(device)]


class Runner:
    """One model (original or patched) bound to its entry."""

    def __init__(self, bundle_dir: Path, patched: bool):
        from ..autotuner_runtime.apply import apply
        self.meta = read_meta(bundle_dir)
        model = build_target(self.meta)
        self.model = apply(model, bundle_dir) if patched else model
        self.entry = ENTRIES[self.meta["entry"]]
        self.state: dict = {}

    def __call__(self, inputs):
        with torch.no_grad():
            return [o.clone() for o in self.entry(self.model, inputs, self.state)]


# ------------------------------------------------------------------ validate
def check_workload(original: Runner, patched: Runner, inputs, meta: dict, label: str) -> dict:
    from ..autotuner_runtime import numeric
    exact = meta.get("correctness_rule", "baseline_tolerance") == "exact"
    tol = meta.get("tolerances")
    override = None if tol is None else (tol["rtol"], tol["atol"])
    ref1, ref2 = original(inputs), original(inputs)
    got1, got2 = patched(inputs), patched(inputs)
    res = {"name": label, "rule": "exact" if exact else "baseline_tolerance", "passed": False, "reason": "",
           "max_abs": None, "cosine": None, "failure": None}
    if [tuple(t.shape) for t in ref1] != [tuple(t.shape) for t in got1] or \
            [t.dtype for t in ref1] != [t.dtype for t in got1]:
        return {**res, "reason": "output structure, shape or dtype changed"}
    for name, a, b in (("original_repeat", ref1, ref2), ("patched_repeat", got1, got2)):
        for k, (x, y) in enumerate(zip(a, b)):
            r = numeric.check(y, x, exact=True)
            if not r.passed:
                return {**res, "reason": f"{name.replace('_', ' ')} is not bitwise repeatable",
                        "failure": {"comparison": name, "output": k, "detail": r.detail}}
    worst, cos = 0.0, 1.0
    for k, (x, y) in enumerate(zip(ref1, got1)):
        rtol, atol = numeric.tolerance_for(x.dtype, override)
        r = numeric.check(y, x, exact=exact, rtol=rtol, atol=atol)
        worst = max(worst, numeric.max_abs_diff(y, x))
        cos = min(cos, numeric.cosine(y, x))
        if not r.passed:
            idx = r.index
            detail = {"comparison": "patched_vs_original", "output": k, "reason": r.reason, "detail": r.detail,
                      "index": None if idx is None else list(idx)}
            if idx is not None:
                detail.update(original=float(x[idx].float()), patched=float(y[idx].float()))
            return {**res, "reason": r.reason, "max_abs": worst, "cosine": cos, "failure": detail}
    return {**res, "passed": True, "max_abs": worst, "cosine": cos}


def validate(bundle_dir, original: Runner | None = None, patched: Runner | None = None) -> list[dict]:
    bundle_dir = Path(bundle_dir)
    meta = read_meta(bundle_dir)
    original = original or Runner(bundle_dir, patched=False)
    patched = patched or Runner(bundle_dir, patched=True)
    return [check_workload(original, patched, workload_inputs(bundle_dir, w), meta, label)
            for label, w in meta["workloads"].items()]


# ------------------------------------------------------------------ benchmark
def benchmark(bundle_dir, steps: int | None = None, pairs: int | None = None) -> dict:
    from ..autotuner_runtime.measure import Session
    from ..autotuner_runtime.sequence import compare_sequences, make_sequence
    bundle_dir = Path(bundle_dir)
    meta = read_meta(bundle_dir)
    final = meta.get("final_benchmark", {})
    original, patched = Runner(bundle_dir, patched=False), Runner(bundle_dir, patched=True)
    checks = validate(bundle_dir, original, patched)
    rows = []
    if all(c["passed"] for c in checks):
        for label, w in meta["workloads"].items():
            inputs = workload_inputs(bundle_dir, w)
            n = steps or final.get("steps", 5)
            base = make_sequence(lambda *a: original(list(a)), inputs, n)
            cand = make_sequence(lambda *a: patched(list(a)), inputs, n)
            row = compare_sequences(Session(), base, cand, pairs=pairs or final.get("pairs", 4),
                                    warmup_steps=final.get("warmup_steps", 3), label=label)
            rows.append({"workload": label, "steps": n, **{k: row[k] for k in (
                "baseline_sequence_ms", "candidate_sequence_ms", "speedup", "win_confirmed",
                "regression_confirmed", "pairs")}})
    return {"bundle": bundle_dir.name, "validate": checks, "benchmark": rows}


# ------------------------------------------------------------------ CLI
def _main(kind: str, argv=None) -> int:
    ap = argparse.ArgumentParser(prog=f"python -m metal_autotune_b200.bundles.{kind}")
    ap.add_argument("bundle", type=Path)
    ap.add_argument("--json", type=Path, help="also write the result here")
    if kind == "benchmark":
        ap.add_argument("--steps", type=int, default=None)
        ap.add_argument("--pairs", type=int, default=None)
    args = ap.parse_args(argv)
    if kind == "validate":
        out = {"bundle": args.bundle.name, "validate": validate(args.bundle)}
        ok = all(c["passed"] for c in out["validate"])
    else:
        out = benchmark(args.bundle, args.steps, args.pairs)
        ok = all(c["passed"] for c in out["validate"]) and bool(out["benchmark"])
    text = json.dumps(out, indent=1, default=float)
    print(text)
    if args.json:
        args.json.write_text(text + "\n")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(_main(sys.argv[1] if len(sys.argv) > 1 else "validate", sys.argv[2:]))
