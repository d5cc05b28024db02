"""Copy grouping (the reference's autotuner/regions/fingerprint.py): two
stretches are copies of one region when their canonical forms agree: the op
sequence with its non-shape arguments, dtypes and ranks, the internal edges,
and the ordered boundary roles, with array identities replaced by roles.
Activation shapes and the shape arguments of views are left out (the same
sequence at another size is the same region); weights count by shape (a
projection against another matrix shape is another kernel).
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict
from dataclasses import dataclass, field

from .build import Stretch, base, is_view, weight_like_ids
from .trace import ArrayRef, Trace


def _canon(obj):
    if isinstance(obj, ArrayRef):
        return ("ref", obj.index)
    if isinstance(obj, (list, tuple)):
        return tuple(_canon(v) for v in obj)
    if isinstance(obj, dict):
        return tuple(sorted((k, _canon(v)) for k, v in obj.items()))
    return repr(obj)


def canonical_form(trace: Trace, s: Stretch, weight_like: frozenset | None = None) -> tuple:
    weight_like = weight_like_ids(trace) if weight_like is None else weight_like
    nodes = trace.nodes[s.start_seq:s.end_seq + 1]
    roles: dict[int, tuple] = {}
    x = w = 0
    form = []
    for pos, node in enumerate(nodes):
        ins = []
        for aid, (shape, _) in zip(node.in_arrays, node.in_specs):
            if aid not in roles:
                if aid in weight_like:
                    roles[aid] = ("w", w, tuple(shape))
                    w += 1
                else:
                    roles[aid] = ("x", x)
                    x += 1
            ins.append(roles[aid])
        for slot, aid in enumerate(node.out_arrays):
            roles[aid] = ("i", pos, slot)
        args = () if is_view(node) else _canon(node.args)
        form.append((node.op if not is_view(node) else base(node.op), args, tuple(ins),
                     tuple((len(sh), dt) for sh, dt in node.out_specs),
                     tuple(dt for _, dt in node.in_specs)))
    return (tuple(form), tuple(roles[a] for a in s.input_ids), tuple(roles[a] for a in s.output_ids))


def fingerprint(form: tuple) -> str:
    return hashlib.sha256(repr(form).encode()).hexdigest()[:16]


@dataclass
class Region:
    fingerprint: str
    ops: tuple                                   # the first copy's op sequence
    members: list = field(default_factory=list)  # Stretches, one per copy
    rejected: str | None = None
    # pricing, per workload (price.py)
    t_orig_ms: dict = field(default_factory=dict)
    t_rep_ms: dict = field(default_factory=dict)
    p: dict = field(default_factory=dict)
    roofline: object = None

    @property
    def copies(self) -> int:
        return len(self.members)

    @property
    def combined_p(self) -> float:
        return sum(self.p.values())

    @property
    def removable_p(self) -> dict:
        """Amdahl's optimistic step reduction p * (1 - 1/s_max) per workload:
        headroom, not a promised win (types.py:78-93)."""
        r = self.roofline
        return {w: max(p, 0.0) * (1.0 - 1.0 / r.s_max) if r is not None and r.s_max > 1.0 else 0.0
                for w, p in self.p.items()}

    @property
    def combined_removable_p(self) -> float:
        return sum(self.removable_p.values())


def group(trace: Trace, stretches: list[Stretch]) -> list[Region]:
    """Regions in order of first appearance, each with all its copies.
    Overlapping copies of one form (a run that repeats inside itself) keep
    the earliest non-overlapping set."""
    wl = weight_like_ids(trace)
    regions: "OrderedDict[str, Region]" = OrderedDict()
    for s in sorted(stretches, key=lambda s: (s.start_seq, s.end_seq)):
        fp = fingerprint(canonical_form(trace, s, wl))
        r = regions.get(fp)
        if r is None:
            r = regions[fp] = Region(fp, tuple(n.op for n in trace.nodes[s.start_seq:s.end_seq + 1]))
        if any(m.start_seq <= s.end_seq and s.start_seq <= m.end_seq for m in r.members):
            continue
        r.members.append(s)
    return list(regions.values())
