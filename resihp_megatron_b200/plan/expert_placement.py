"""Expert placement for resilient expert parallelism (EPLB / Lazarus style).

Within every EP group each logical expert has at least one physical copy; spare slots
replicate the experts with the highest load per copy.  Copies are packed onto devices
most-constrained first (experts with more copies, then heavier copies), never two copies of one
expert on a device, each to the device whose speed-normalised work stays lowest -- except that a
device which already held the expert keeps it while its work stays within ``stickiness`` of its
speed share, so a re-placement moves little expert state.  The slot budget (how many copies in
total) is searched; a budget is scored by the slowest device's expert time when every expert's
tokens split across its holders in proportion to speed, then by copies moved, then by copies.

An expert's gradient sums over all its holders, so expert-data-parallel groups follow from the
placement (``expert_dp_groups``); tokens of a replicated expert are dealt to its holders by
smooth weighted round robin (the nginx upstream balancing rule), deterministic on every rank.
Parity: ``resihp/plan/expert_placement.py:21-168`` (same placement rules, JSON and token split).
"""

from __future__ import annotations

import heapq
import math
from collections import defaultdict
from dataclasses import dataclass

from .planner import PlanInfeasible

_FLOOR = 1e-9


@dataclass(frozen=True)
class ExpertPlacement:
    num_experts: int
    groups: tuple[tuple[str, ...], ...]
    slots: dict[str, tuple[int, ...]]

    def holders(self, expert: int) -> list[str]:
        """Every device (in any group) hosting a copy of ``expert``, sorted."""
        return sorted(d for d, hosted in self.slots.items() if expert in hosted and self._placed(d))

    def _placed(self, device: str) -> bool:
        return any(device in g for g in self.groups)

    def group_holders(self, group: int, expert: int) -> list[str]:
        return [d for d in self.groups[group] if expert in self.slots[d]]

    def group_of(self, device: str) -> int:
        found = [i for i, g in enumerate(self.groups) if device in g]
        if not found:
            raise KeyError(device)
        return found[0]

    def validate(self) -> None:
        want = frozenset(range(self.num_experts))
        for i, g in enumerate(self.groups):
            lacking = want.difference(e for d in g for e in self.slots[d])
            if lacking:
                raise ValueError(f"EP group {i} misses experts {sorted(lacking)}")
            doubled = [d for d in g if len(self.slots[d]) != len(frozenset(self.slots[d]))]
            if doubled:
                raise ValueError(f"{doubled[0]} hosts duplicate copies")

    def to_json(self) -> dict:
        return {"num_experts": self.num_experts, "groups": [list(g) for g in self.groups],
                "slots": {d: list(es) for d, es in self.slots.items()}}

    @classmethod
    def from_json(cls, d: dict) -> "ExpertPlacement":
        return cls(d["num_experts"], tuple(map(tuple, d["groups"])), {k: tuple(v) for k, v in d["slots"].items()})


def replica_counts(loads: list[float], total_slots: int, max_copies: int | None = None) -> list[int]:
    """Copies per expert for ``total_slots`` slots: one each, then every spare slot to the expert
    with the highest load per copy (lower id on ties), at most ``max_copies`` each."""
    E = len(loads)
    if total_slots < E:
        raise PlanInfeasible(f"{total_slots} slots cannot host {E} experts")
    limit = max_copies or total_slots
    counts = [1] * E
    heap = [(-loads[e], e) for e in range(E) if limit > 1]  # key: -(load per copy), then id
    heapq.heapify(heap)
    for _ in range(total_slots - E):
        if not heap:
            break
        _, e = heapq.heappop(heap)
        counts[e] += 1
        if counts[e] < limit:
            heapq.heappush(heap, (-loads[e] / counts[e], e))
    return counts


def group_time(slots: dict[str, tuple[int, ...]], loads: list[float], speeds: dict[str, float]) -> float:
    """The slowest device's expert time when each expert's tokens split across its holders in
    proportion to speed: every holder of ``e`` spends ``load_e / (sum of its holders' speeds)``."""
    pooled: dict[int, float] = defaultdict(float)
    for d, hosted in slots.items():
        for e in hosted:
            pooled[e] += max(speeds.get(d, 1.0), _FLOOR)
    per_device = [sum(loads[e] / pooled[e] for e in hosted) for hosted in slots.values()]
    return max(per_device, default=0.0)


class _Packer:
    """Greedy packing of one budget's copies onto one EP group's devices."""

    def __init__(self, devices, speed, per_device, prev, stickiness):
        self.devices, self.speed, self.cap = devices, speed, per_device
        self.prev, self.slack = prev, 1.0 + stickiness

    def pack(self, loads, counts):
        copies = [(counts[e], loads[e] / counts[e], e) for e in range(len(loads)) for _ in range(counts[e])]
        copies.sort(key=lambda c: (-c[0], -c[1], c[2]))
        total_speed = sum(self.speed.values())
        total_work = sum(w for _, w, _ in copies)
        share = {d: total_work * self.speed[d] / total_speed for d in self.devices}
        hosted = {d: [] for d in self.devices}
        work = dict.fromkeys(self.devices, 0.0)
        for _, w, e in copies:
            open_ = [d for d in self.devices if len(hosted[d]) < self.cap and e not in hosted[d]]
            if not open_:
                return None
            keepers = [d for d in open_ if e in self.prev.get(d, ()) and work[d] + w <= share[d] * self.slack + 1e-12]
            dest = min(keepers or open_, key=lambda d: ((work[d] + w) / self.speed[d], d))
            hosted[dest].append(e)
            work[dest] += w
        return {d: tuple(sorted(es)) for d, es in hosted.items()}


def place_group(devices: list[str], speeds: dict[str, float], loads: list[float], slots_per_device: int,
                prev: dict[str, tuple[int, ...]] | None = None, stickiness: float = 0.1) -> dict[str, tuple[int, ...]]:
    """Slots of one EP group's devices (see the module docstring)."""
    before = prev or {}
    speed = {d: max(speeds.get(d, 1.0), _FLOOR) for d in devices}
    packer = _Packer(devices, speed, slots_per_device, before, stickiness)
    scored = []
    for budget in range(len(loads), len(devices) * slots_per_device + 1):
        slots = packer.pack(loads, replica_counts(loads, budget, max_copies=len(devices)))
        if slots is None:
            continue
        fresh = sum(e not in before.get(d, ()) for d, es in slots.items() for e in es)
        scored.append(((round(group_time(slots, loads, speed), 12), fresh, budget), slots))
    if not scored:
        raise PlanInfeasible(f"cannot place {len(loads)} experts on {len(devices)} devices x {slots_per_device}")
    return min(scored, key=lambda t: t[0])[1]


def plan_expert_placement(ep_groups: list[list[str]], num_experts: int, *, speeds: dict[str, float] | None = None,
                          loads: list[float] | None = None, prev: ExpertPlacement | None = None,
                          max_slots: int | None = None, slots_per_device: int | None = None) -> ExpertPlacement:
    """Placement over several EP groups (each hosts every expert), validated."""
    load = list(loads) if loads else [1.0] * num_experts
    earlier = prev.slots if prev else {}
    slots: dict[str, tuple[int, ...]] = {}
    for g in ep_groups:
        if max_slots is not None and len(g) * max_slots < num_experts:
            raise PlanInfeasible(f"EP group of {len(g)} devices x {max_slots} slots cannot host {num_experts}")
        per_device = slots_per_device or math.ceil(num_experts / len(g))
        if max_slots is not None:
            per_device = min(per_device, max_slots)
        slots |= place_group(list(g), speeds or {}, load, per_device, earlier)
    placement = ExpertPlacement(num_experts, tuple(map(tuple, ep_groups)), slots)
    placement.validate()
    return placement


def expert_dp_groups(placement: ExpertPlacement) -> dict[tuple[str, ...], list[int]]:
    """Experts with identical holder sets share one gradient all-reduce group."""
    by_holders: dict[tuple[str, ...], list[int]] = {}
    for e in range(placement.num_experts):
        by_holders.setdefault(tuple(placement.holders(e)), []).append(e)
    return by_holders


def smooth_weighted_round_robin(holders: list[str], speeds: dict[str, float], n: int) -> list[str]:
    """Deal ``n`` tokens of an expert to its replicas in proportion to speed, interleaved.

    Smooth weighted round robin (integer weights ``round(10 * speed)``, at least 1): every turn
    each replica's credit grows by its weight, the replica with the most credit (larger name on
    ties) takes the token and pays back the total weight."""
    if len(holders) == 1:
        return [holders[0]] * n
    weight = [max(1, round(10 * speeds.get(h, 1.0))) for h in holders]
    total = sum(weight)
    credit = [0] * len(holders)
    dealt = []
    for _ in range(n):
        credit = [c + w for c, w in zip(credit, weight)]
        k = max(range(len(holders)), key=lambda i: (credit[i], holders[i]))
        credit[k] -= total
        dealt.append(holders[k])
    return dealt


def moved_experts(old: ExpertPlacement, new: ExpertPlacement) -> int:
    """Copies in ``new`` that their device did not hold in ``old``."""
    return sum(e not in old.slots.get(d, ()) for d, hosted in new.slots.items() for e in hosted)
