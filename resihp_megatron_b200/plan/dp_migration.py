"""Progress-aware stage-level micro-batch migration across DP replicas (ResiHP Algorithm 1).

Micro-batch ``m`` of (virtual) stage ``s`` runs on replica ``assignment[s][m]``.  The search:

1. **Starting points.**  The given assignment, an ``equal`` split and a ``speed``-weighted split
   (largest-remainder shares by each replica's slowest stage; a stage a replica lost is taken
   over, micro-batch by micro-batch, by the surviving replica with the least speed-normalised
   load).  The one the simulator predicts fastest (and within the memory caps) is kept.
2. **Steepest descent.**  In each round, on every physical stage with two or more replicas, the
   replica that finishes its forwards last hands its last forward micro-batch to the one that
   finishes first -- offered both as a *stage* move (that stage only, every virtual chunk of it)
   and as a *pipeline* move (every stage where the receiver has a group).  Every offer is
   simulated; the best is applied if it shortens the makespan without deadlock and keeps every
   slot's in-flight peak under its cap.  The search stops when no offer improves.

Parity: ``resihp/plan/dp_migration.py:32-147`` (same starting points, moves and acceptance rule).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from fractions import Fraction
from typing import Callable

from .cost_model import CostModel
from .hetero_plan import HeteroParallelPlan, StageGroup
from .simulator import SimResult, schedule_with_fallback

Key = tuple[int, int]
_EPS = 1e-12


@dataclass
class MigrationResult:
    assignment: tuple[tuple[int, ...], ...]
    makespan: float
    moves: int
    sim: SimResult
    initial_makespan: float


def simulate(plan: HeteroParallelPlan, cm: CostModel, split_backward: bool = False) -> SimResult:
    """Pipeline simulation of ``plan`` priced by ``cm`` (best of the available schedules)."""
    return schedule_with_fallback(plan, cm.cost, cm.comm, split_backward=split_backward, sync_time=cm.sync_time)


def largest_remainder(total: int, weights: list[float]) -> list[int]:
    """Integer shares of ``total`` proportional to ``weights``: floors first, then one more for
    the largest fractional remainders (lower index first on ties)."""
    whole = sum(weights)
    exact = [Fraction(total) * Fraction(w) / Fraction(whole) for w in weights]
    shares = [math.floor(q) for q in exact]
    by_remainder = sorted(range(len(weights)), key=lambda i: (shares[i] - exact[i], i))
    for i in by_remainder[:total - sum(shares)]:
        shares[i] += 1
    return shares


def initial_assignment(groups: list[StageGroup], num_stages: int, num_microbatches: int,
                       speed: Callable[[Key], float], mode: str = "speed") -> tuple[tuple[int, ...], ...]:
    """A stage-major assignment: the same replica split on every stage, patched on stages a
    replica lost by handing its micro-batches to the survivor with the least relative load."""
    present = {(g.replica, g.stage) for g in groups}
    replicas = sorted({g.replica for g in groups})

    def weight(r: int) -> float:
        if mode == "equal":
            return 1.0
        return min(speed((r, s)) for s in range(num_stages) if (r, s) in present)

    shares = largest_remainder(num_microbatches, [weight(r) for r in replicas])
    template = [r for r, n in zip(replicas, shares) for _ in range(n)]
    table = []
    for s in range(num_stages):
        owners = [r for r in replicas if (r, s) in present]
        count = {r: template.count(r) for r in owners}
        row = []
        for r in template:
            if r not in count:  # the replica lost this stage
                r = min(owners, key=lambda x: ((count[x] + 1) / max(speed((x, s)), _EPS), x))
                count[r] += 1
            row.append(r)
        table.append(tuple(row))
    return tuple(table)


class _Descent:
    def __init__(self, cm: CostModel, mem_cap, split_backward: bool, delta: float):
        self.cm, self.caps, self.split, self.delta = cm, mem_cap, split_backward, delta

    def run(self, plan: HeteroParallelPlan) -> SimResult:
        return simulate(plan, self.cm, self.split)

    def acceptable(self, res: SimResult) -> bool:
        if res.deadlock:
            return False
        return self.caps is None or all(n <= self.caps.get(k, math.inf) for k, n in res.peak_inflight.items())

    def offers(self, plan: HeteroParallelPlan, sim: SimResult):
        seen = []
        for s in range(plan.num_physical_stages):
            replicas = [g.replica for g in plan.groups_at(s)]
            if len(replicas) < 2:
                continue
            finish = {r: sim.stage_forward_done.get((r, s), 0.0) for r in replicas}
            ranked = sorted(replicas, key=lambda r: (finish[r], r))
            fast, slow = ranked[0], max(replicas, key=lambda r: (finish[r], -r))
            if fast == slow or finish[slow] - finish[fast] <= self.delta:
                continue
            forwards = [e[1] for e in sim.order[(slow, s)] if e[0] == "F" and (len(e) == 2 or e[2] == s)]
            if len(forwards) < 2:
                continue
            for offer in (("stage", s, forwards[-1], slow, fast), ("pipeline", -1, forwards[-1], slow, fast)):
                if offer not in seen:
                    seen.append(offer)
        return seen

    @staticmethod
    def apply(plan: HeteroParallelPlan, kind: str, s: int, m: int, slow: int, fast: int) -> HeteroParallelPlan:
        table = [list(row) for row in plan.assignment]
        if kind == "stage":  # every virtual chunk of physical stage s
            targets = range(s, plan.num_stages, plan.num_physical_stages)
        else:
            targets = [t for t in range(plan.num_stages) if table[t][m] == slow and plan.group(fast, t) is not None]
        for t in targets:
            table[t][m] = fast
        return replace(plan, assignment=tuple(map(tuple, table)))


def progress_aware_migration(plan: HeteroParallelPlan, cm: CostModel, *, mem_cap: dict[Key, float] | None = None,
                             delta: float = 0.0, max_rounds: int = 32, split_backward: bool = False) -> MigrationResult:
    search = _Descent(cm, mem_cap, split_backward, delta)
    given = search.run(plan)
    starts = [(given.makespan, "given", plan)]
    for mode in ("equal", "speed"):
        table = initial_assignment(list(plan.stage_groups), plan.num_stages, plan.num_microbatches,
                                   cm.group_speed, mode)
        candidate = replace(plan, assignment=table)
        res = search.run(candidate)
        if search.acceptable(res):
            starts.append((res.makespan, mode, candidate))
    current = min(starts, key=lambda t: (t[0], t[1]))[2]
    sim = search.run(current)
    applied = 0
    while applied < max_rounds:
        winner = None
        for offer in search.offers(current, sim):
            trial = search.apply(current, *offer)
            if trial.assignment == current.assignment:
                continue
            res = search.run(trial)
            bar = winner[1].makespan if winner else sim.makespan
            if search.acceptable(res) and res.makespan < bar - _EPS:
                winner = (trial, res)
        if winner is None:
            break
        current, sim = winner
        applied += 1
    return MigrationResult(current.assignment, sim.makespan, applied, sim, given.makespan)
