"""Slice-level state-transfer planning between two plans.

For every interval a device must hold in the new plan: the parts it already holds (from a
valid, up-to-date source) are reused in place; the rest is cut at the boundaries of the
surviving holders and each piece gets the closest, least-loaded source (same node < same rack
< other, then bytes already assigned, then name), optionally striped in chunks so large moves
spread over DP replicas; pieces with no valid holder are reported as lost (fallback to
snapshots / checkpoints).  Every rank computes the identical plan from identical inputs -- no
coordinator round trip.  (Reference: ``resihp/state/transfer_plan.py:23-106``.)
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field

from .layer_registry import Holdings, TensorSpec
from ..utils.intervals import intersect


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
        total = 0
        for t in self.transfers:
            s = specs[t.key]
            n = 1
            for d in s.local_shape(t.interval):
                n *= d
            total += n * bytes_per_elem * (kinds if s.trainable else 1)
        return total


def subtract(iv: tuple[int, int], cuts: list[tuple[int, int]]) -> list[tuple[int, int]]:
    """``iv`` minus the union of ``cuts`` as a list of intervals."""
    rest = [iv]
    for c in cuts:
        nxt = []
        for a in rest:
            o = intersect(a, c)
            if o is None:
                nxt.append(a)
                continue
            if a[0] < o[0]:
                nxt.append((a[0], o[0]))
            if o[1] < a[1]:
                nxt.append((o[1], a[1]))
        rest = nxt
    return rest


def plan_transfers(old: Holdings, new: Holdings, *, valid_sources: set[str], node_of: dict[str, str],
                   rack_of: dict[str, str] | None = None, chunk: int | None = None) -> TransferPlan:
    rack_of = rack_of or {}
    plan = TransferPlan()
    load: dict[str, int] = defaultdict(int)

    def distance(src: str, dst: str) -> int:
        if node_of.get(src) == node_of.get(dst):
            return 0
        if rack_of.get(src) is not None and rack_of.get(src) == rack_of.get(dst):
            return 1
        return 2

    for key in sorted(new):
        sources = [(d, iv) for d, iv in old.get(key, []) if d in valid_sources]
        for dst, want in sorted(new[key]):
            mine = [iv for d, iv in sources if d == dst]
            for iv in mine:
                o = intersect(iv, want)
                if o is not None:
                    plan.reuse.append((dst, key, o))
            for gap in subtract(want, mine):
                holders = [(d, iv) for d, iv in sources if d != dst and intersect(iv, gap) is not None]
                cuts = {gap[0], gap[1]}
                for _, iv in holders:
                    cuts.update(x for x in iv if gap[0] < x < gap[1])
                pts = sorted(cuts)
                for piece in zip(pts, pts[1:]):
                    cands = sorted({d for d, iv in holders if iv[0] <= piece[0] and piece[1] <= iv[1]})
                    if not cands:
                        plan.lost.append((key, piece))
                        continue
                    if chunk and piece[1] - piece[0] > chunk:
                        pieces = [(a, min(a + chunk, piece[1])) for a in range(piece[0], piece[1], chunk)]
                    else:
                        pieces = [piece]
                    for p in pieces:
                        src = min(cands, key=lambda d: (distance(d, dst), load[d], d))
                        load[src] += p[1] - p[0]
                        plan.transfers.append(SliceTransfer(key, src, dst, p))
    plan.transfers.sort(key=lambda t: (t.key, t.interval, t.src, t.dst))
    plan.load = dict(load)
    return plan
