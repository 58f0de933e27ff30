"""Slice-level planning of the state transfers between two plans.

For every interval a device must hold under the new plan: the parts it already holds (as a
valid, up-to-date source) are reused in place.  The rest is swept left to right over the
boundaries of the valid holders, giving pieces that each lie inside one or more holders'
intervals; every piece (optionally cut into ``chunk``-sized spans so a large move stripes over
the DP replicas) is read from the closest, least-loaded holder -- same node before same rack
before anywhere, then fewer elements already assigned, then the name.  Pieces nobody valid
holds are reported as lost (the caller falls back to snapshots or checkpoints).  Every rank
computes the identical plan from identical inputs, so no coordinator round trip is needed.
Parity: ``resihp/state/transfer_plan.py:23-106`` (same reuse, locality and striping rules).
"""

from __future__ import annotations

import math
from collections import defaultdict
from dataclasses import dataclass, field

from .layer_registry import Holdings, TensorSpec
from ..utils.intervals import intersect

Interval = tuple[int, int]


@dataclass(frozen=True)
class SliceTransfer:
    key: str
    src: str
    dst: str
    interval: tuple[int, int]


@dataclass
class TransferPlan:
    transfers: list[SliceTransfer] = field(default_factory=list)
    reuse: list[tuple[str, str, tuple[int, int]]] = field(default_factory=list)
    lost: list[tuple[str, tuple[int, int]]] = field(default_factory=list)
    load: dict[str, int] = field(default_factory=dict)

    def bytes_moved(self, specs: dict[str, TensorSpec], bytes_per_elem: int, kinds: int) -> int:
        """Bytes on the wire when each trainable tensor moves ``kinds`` copies (value, moments)."""
        return sum(math.prod(specs[t.key].local_shape(t.interval)) * bytes_per_elem *
                   (kinds if specs[t.key].trainable else 1) for t in self.transfers)


def subtract(iv: tuple[int, int], cuts: list[tuple[int, int]]) -> list[tuple[int, int]]:
    """``iv`` minus the union of ``cuts``, as ordered disjoint intervals."""
    lo, hi = iv
    covered = sorted(c for c in (intersect(iv, c) for c in cuts) if c is not None)
    remaining, at = [], lo
    for a, b in covered:
        if a > at:
            remaining.append((at, a))
        at = max(at, b)
    if at < hi:
        remaining.append((at, hi))
    return remaining


def _pieces(gap: Interval, holders: list[tuple[str, Interval]]):
    """Sweep ``gap`` at every holder boundary inside it; yields ``(piece, covering holders)``."""
    edges = sorted({gap[0], gap[1], *(x for _, iv in holders for x in iv if gap[0] < x < gap[1])})
    for a, b in zip(edges, edges[1:]):
        yield (a, b), sorted({d for d, (lo, hi) in holders if lo <= a and b <= hi})


def _spans(piece: Interval, chunk: int | None):
    a, b = piece
    if not chunk or b - a <= chunk:
        return [piece]
    return [(s, min(s + chunk, b)) for s in range(a, b, chunk)]


class _SourcePicker:
    def __init__(self, node_of: dict[str, str], rack_of: dict[str, str]):
        self.node_of, self.rack_of = node_of, rack_of
        self.load: dict[str, int] = defaultdict(int)

    def _distance(self, src: str, dst: str) -> int:
        if self.node_of.get(src) == self.node_of.get(dst):
            return 0
        rack = self.rack_of.get(src)
        return 1 if rack is not None and rack == self.rack_of.get(dst) else 2

    def pick(self, candidates: list[str], dst: str, span: Interval) -> str:
        src = min(candidates, key=lambda d: (self._distance(d, dst), self.load[d], d))
        self.load[src] += span[1] - span[0]
        return src


def plan_transfers(old: Holdings, new: Holdings, *, valid_sources: set[str], node_of: dict[str, str],
                   rack_of: dict[str, str] | None = None, chunk: int | None = None) -> TransferPlan:
    plan = TransferPlan()
    picker = _SourcePicker(node_of, rack_of or {})
    for key in sorted(new):
        valid = [(d, iv) for d, iv in old.get(key, []) if d in valid_sources]
        for dst, want in sorted(new[key]):
            own = [iv for d, iv in valid if d == dst]
            plan.reuse.extend((dst, key, o) for o in (intersect(iv, want) for iv in own) if o is not None)
            for gap in subtract(want, own):
                holders = [(d, iv) for d, iv in valid if d != dst and intersect(iv, gap) is not None]
                for piece, covering in _pieces(gap, holders):
                    if not covering:
                        plan.lost.append((key, piece))
                        continue
                    for span in _spans(piece, chunk):
                        plan.transfers.append(SliceTransfer(key, picker.pick(covering, dst, span), dst, span))
    plan.transfers.sort(key=lambda t: (t.key, t.interval, t.src, t.dst))
    plan.load = dict(picker.load)
    return plan
