"""Exact tensor comparison including signed zeros and NaN payloads (the
reference's autotuner_runtime/exact.py:5-10), by the GPU diff reduction's
bit-pattern count."""
from __future__ import annotations

import torch


def bitwise_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    if tuple(a.shape) != tuple(b.shape) or a.dtype != b.dtype:
        return False
    if a.numel() == 0:
        return True
    from .numeric import diff_stats
    return diff_stats(a, b).bit_mismatches == 0
