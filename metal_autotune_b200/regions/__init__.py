"""Region discovery for torch models: record a step's aten op stream
(trace.py), cut it into candidate stretches (build.py), group copies by
canonical form (fingerprint.py), bound each by its roofline (roofline.py),
price it on the GPU with CUDA events (price.py) and rank by the step time
an ideal kernel could remove (rank.py). The reference's autotuner/trace/ and
autotuner/regions/ (build.py:128, fingerprint.py, roofline.py:75,
price.py:209, rank.py) do this for MLX models on Apple GPUs.

    trace, regions = discover(model, (x,), "whisper_tiny")
    step_ms = price.price(trace, regions, model, (x,), roofline.peaks())   # GPU
    for r in rank.rank(rank.apply_floor(regions)): ...

`python -m metal_autotune_b200.regions <target> [--price]` prints the table.
"""
from __future__ import annotations

from . import build, fingerprint, price, rank, roofline, trace
from .fingerprint import Region
from .trace import Trace

__all__ = ["discover", "pattern_fingerprint", "build", "fingerprint", "price", "rank", "roofline", "trace", "Region",
           "Trace"]


def discover(module, args: tuple, workload: str = "step") -> tuple[Trace, list[Region]]:
    """The recorded trace of module(*args) and its candidate regions, each
    with every copy found (no GPU needed: the trace runs on fake tensors)."""
    t = trace.record(module, args, workload)
    return t, fingerprint.group(t, build.build_stretches(t))


class _Pattern:
    """A region's original-op function as a module: the inputs at `weights`
    positions are its buffers (weights to the fingerprint), the rest its
    arguments."""

    @staticmethod
    def make(fn, inputs, weights):
        import torch.nn as nn

        class P(nn.Module):
            def __init__(self):
                super().__init__()
                for i in weights:
                    self.register_buffer(f"w{i}", inputs[i])

            def forward(self, *acts):
                it = iter(acts)
                return fn(*[getattr(self, f"w{i}") if i in weights else next(it) for i in range(len(inputs))])
        return P(), tuple(inputs[i] for i in range(len(inputs)) if i not in weights)


def pattern_fingerprint(fn, inputs, weights=()) -> str:
    """Fingerprint of the stretch made of all of fn's calls on these inputs
    (the positions in `weights` count as weights): the region a discovered
    copy of this pattern groups under."""
    module, args = _Pattern.make(fn, list(inputs), set(weights))
    t = trace.record(module, args, "pattern")
    s = build.boundary(t, 0, len(t.nodes) - 1)
    return fingerprint.fingerprint(fingerprint.canonical_form(t, s))
