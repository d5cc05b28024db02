"""python -m metal_autotune_b200.regions <target> [--price] [--top N] [--json FILE]

Discovers the candidate regions of one target's step (its seeded random
model and workload input) and prints them: copies, ops, boundary bytes,
roofline; with --price (GPU) the measured one-copy time, the share p of the
step, s_max and the removable share p(1 - 1/s_max), ranked."""
from __future__ import annotations

import argparse
import json

import torch

from . import discover, price, rank, roofline
from .build import base, is_view

TARGETS = ("tiny_mlp", "whisper_tiny", "whisper_turbo", "mamba_tiny", "qwen3_tiny_prefill")


def target(name: str, device: str):
    from ..targets import mamba, qwen3, tiny_mlp, whisper
    if name == "tiny_mlp":
        m, x = tiny_mlp.build(device=device)
        return m, (x,)
    if name.startswith("whisper"):
        cfg = whisper.TINY if name == "whisper_tiny" else whisper.WHISPER_TURBO
        g = torch.Generator(device=device).manual_seed(0)
        x = torch.randn(2 if cfg is whisper.TINY else 1, cfg.frames, cfg.n_mels, generator=g, device=device)
        return whisper.build(cfg, seed=0, device=device), (x.to(torch.float16),)
    if name == "mamba_tiny":
        from .. import workload
        m = mamba.build(mamba.TINY, seed=0, device=device)
        return m, (workload.seeded_tokens((64,), 0, mamba.TINY.vocab, seed=0, device=device),)
    if name == "qwen3_tiny_prefill":
        from .. import workload
        m = qwen3.build(qwen3.TINY, seed=0, device=device)
        return _Qwen3Prefill(m), (workload.seeded_tokens((32,), 0, qwen3.TINY.vocab, seed=0, device=device),)
    raise SystemExit(f"unknown target {name}; one of {', '.join(TARGETS)}")


class _Qwen3Prefill(torch.nn.Module):
    """Qwen3 prefill from an empty cache as one step."""

    def __init__(self, model):
        super().__init__()
        self.model = model

    def forward(self, tokens):
        from ..targets import qwen3
        cache = qwen3.KVCache(self.model.cfg, device=tokens.device)
        return self.model(tokens, cache)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("target", choices=TARGETS)
    ap.add_argument("--price", action="store_true", help="time regions and the step on the GPU")
    ap.add_argument("--top", type=int, default=15)
    ap.add_argument("--json", default="")
    a = ap.parse_args()
    device = "cuda" if a.price else "cpu"
    model, args = target(a.target, device)
    trace, regions = discover(model, args, a.target)
    pk = roofline.peaks()
    rows = []
    est = price.estimate(trace, regions, pk)
    wave, deferred = rank.select_frontier(regions, lambda r: est[r.fingerprint][1])
    if a.price:  # the non-overlapping wave is priced; the deferred alternatives wait behind it
        step_ms = price.price(trace, wave, model, args, pk)
        kept = rank.rank(rank.apply_floor(wave))
    else:
        step_ms, kept = None, wave
    floor = roofline.step_floor(trace, pk, step_ms or 0.0)
    for r in kept[: a.top]:
        s = r.members[0]
        roof = r.roofline or roofline.stretch_roofline(trace, s, pk)
        row = {"fingerprint": r.fingerprint, "copies": r.copies, "scope": s.scope_stack[-1],
               "ops": [base(o) for o in r.ops if not is_view(type("N", (), {"op": o})())],
               "bound": roof.bound, "t_roofline_us": round(roof.t_roofline_ms * 1e3, 2)}
        if a.price:
            row.update({"t_copy_us": round(r.t_rep_ms[a.target] * 1e3, 2), "p": round(r.combined_p, 4),
                        "s_max": round(roof.s_max, 2), "removable_p": round(r.combined_removable_p, 4)})
        rows.append(row)
        print(json.dumps(row))
    summary = {"target": a.target, "calls": len(trace.nodes), "regions": len(regions), "wave": len(wave),
               "deferred": len(deferred), "priced": bool(a.price), "peaks": pk.source, "step_floor": floor}
    print(json.dumps(summary))
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"summary": summary, "ranked": rows}, f, indent=1)


if __name__ == "__main__":
    main()
