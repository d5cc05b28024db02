"""Which regions to work on first (the reference's autotuner/regions/rank.py):
drop copies-together shares under a floor, then order by the step time an
ideal kernel could remove, p * (1 - 1/s_max) (Amdahl: step speed-up
1 / (1 - p + p/s) orders the same way), weighted down 1% per op beyond the
first (a longer kernel is harder to write); and pick a non-overlapping wave
of candidates to price first, the rest deferred behind the cut they overlap.
"""
from __future__ import annotations

from .build import VIEW_OPS, base
from .fingerprint import Region

REGION_FLOOR_P = 0.02
LENGTH_PENALTY = 0.01
_BOUND_ORDER = {"memory": 0, "launch": 1, "compute": 2}


def length_weight(region: Region) -> float:
    ops = sum(base(op) not in VIEW_OPS for op in region.ops)
    return max(0.0, 1.0 - LENGTH_PENALTY * (max(ops, 1) - 1))


def apply_floor(regions: list[Region], floor: float = REGION_FLOOR_P) -> list[Region]:
    """Keep priced regions whose copies together reach `floor` of the step;
    mark the others with the reason (rank.py:53-66)."""
    kept = []
    for r in regions:
        if r.rejected:
            continue
        if r.combined_p < floor:
            r.rejected = f"under floor: combined p {r.combined_p:.4f} < {floor}"
        else:
            kept.append(r)
    return kept


def rank(regions: list[Region]) -> list[Region]:
    return sorted(regions, key=lambda r: (-r.combined_removable_p * length_weight(r), -r.combined_p,
                                          _BOUND_ORDER.get(r.roofline.bound if r.roofline else "compute", 3),
                                          r.fingerprint))


def _overlap(a: Region, b: Region) -> bool:
    return any(x.workload == y.workload and x.start_seq <= y.end_seq and y.start_seq <= x.end_seq
               for x in a.members for y in b.members)


def select_frontier(regions: list[Region], score) -> tuple[list[Region], dict]:
    """Non-overlapping wave in score order; every other candidate is deferred
    behind the selected cuts it overlaps (rank.py:150-178)."""
    ready, deferred = [], {}
    for r in sorted((r for r in regions if not r.rejected), key=lambda r: (-score(r), len(r.ops), r.fingerprint)):
        conflicts = [c.fingerprint for c in ready if _overlap(r, c)]
        if conflicts:
            deferred[r.fingerprint] = conflicts
        else:
            ready.append(r)
    return ready, deferred
