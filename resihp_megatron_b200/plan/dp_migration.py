"""Progress-aware stage-level micro-batch migration across DP replicas (ResiHP Algorithm 1).

Start from the best of the given assignment, an ``equal`` split and a ``speed``-weighted split
(largest-remainder rounding over each replica's slowest available stage; micro-batches of a
stage a replica lost go to the least-loaded surviving replica of that stage).  Then steepest
descent: at every stage with >= 2 replicas, take the last forward of the replica that finishes
its forwards latest and offer it to the replica that finishes first -- as a *stage* move (one
stage of one micro-batch) and as a *pipeline* move (that micro-batch on every stage where the
fast replica exists).  Each move is simulated; the best one is kept only if the makespan drops
and every slot's in-flight peak stays under its memory cap.
(Reference: ``resihp/plan/dp_migration.py:32-147``.)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Callable

from .cost_model import CostModel
from .hetero_plan import HeteroParallelPlan, StageGroup
from .simulator import SimResult, schedule_with_fallback

Key = tuple[int, int]


@dataclass
class MigrationResult:
    assignment: tuple[tuple[int, ...], ...]
    makespan: float
    moves: int
    sim: SimResult
    initial_makespan: float


def simulate(plan: HeteroParallelPlan, cm: CostModel, split_backward: bool = False) -> SimResult:
    return schedule_with_fallback(plan, cm.cost, cm.comm, split_backward=split_backward, sync_time=cm.sync_time)


def largest_remainder(total: int, weights: list[float]) -> list[int]:
    """Integer shares of ``total`` proportional to ``weights`` (largest remainder, ties by index)."""
    s = sum(weights)
    quotas = [total * w / s for w in weights]
    counts = [int(q) for q in quotas]
    short = total - sum(counts)
    for i in sorted(range(len(weights)), key=lambda i: (-(quotas[i] - counts[i]), i))[:short]:
        counts[i] += 1
    return counts


def initial_assignment(groups: list[StageGroup], num_stages: int, num_microbatches: int,
                       speed: Callable[[Key], float], mode: str = "speed") -> tuple[tuple[int, ...], ...]:
    avail = {(g.replica, g.stage) for g in groups}
    replicas = sorted({g.replica for g in groups})
    if mode == "equal":
        w = [1.0] * len(replicas)
    else:
        w = [min(speed((r, s)) for s in range(num_stages) if (r, s) in avail) for r in replicas]
    base: list[int] = []
    for r, c in zip(replicas, largest_remainder(num_microbatches, w)):
        base += [r] * c
    rows = []
    for s in range(num_stages):
        here = [r for r in replicas if (r, s) in avail]
        row = list(base)
        load = {r: row.count(r) for r in here}
        for m, r in enumerate(row):
            if r not in load:  # this replica lost stage s: evict to the least-loaded survivor
                dst = min(here, key=lambda x: ((load[x] + 1) / max(speed((x, s)), 1e-12), x))
                row[m] = dst
                load[dst] += 1
        rows.append(tuple(row))
    return tuple(rows)


def _move(plan: HeteroParallelPlan, kind: str, s: int, m: int, slow: int, fast: int) -> HeteroParallelPlan:
    rows = [list(r) for r in plan.assignment]
    if kind == "stage":
        for t in range(s, plan.num_stages, plan.num_physical_stages):
            rows[t][m] = fast
    else:
        for t in range(plan.num_stages):
            if rows[t][m] == slow and plan.group(fast, t) is not None:
                rows[t][m] = fast
    return replace(plan, assignment=tuple(tuple(r) for r in rows))


def progress_aware_migration(plan: HeteroParallelPlan, cm: CostModel, *, mem_cap: dict[Key, float] | None = None,
                             delta: float = 0.0, max_rounds: int = 32, split_backward: bool = False) -> MigrationResult:
    def within_caps(res: SimResult) -> bool:
        return mem_cap is None or all(v <= mem_cap.get(k, math.inf) for k, v in res.peak_inflight.items())

    given = simulate(plan, cm, split_backward)
    starts = [(given.makespan, "given", plan)]
    for mode in ("equal", "speed"):
        cand = replace(plan, assignment=initial_assignment(list(plan.stage_groups), plan.num_stages,
                                                           plan.num_microbatches, cm.group_speed, mode))
        res = simulate(cand, cm, split_backward)
        if not res.deadlock and within_caps(res):
            starts.append((res.makespan, mode, cand))
    cur = min(starts, key=lambda t: (t[0], t[1]))[2]
    sim = simulate(cur, cm, split_backward)
    moves = 0
    for _ in range(max_rounds):
        offers = []
        for s in range(cur.num_physical_stages):
            gs = cur.groups_at(s)
            if len(gs) < 2:
                continue
            done = {g.replica: sim.stage_forward_done.get((g.replica, s), 0.0) for g in gs}
            slow = max(done, key=lambda r: (done[r], -r))
            fast = min(done, key=lambda r: (done[r], r))
            if slow == fast or done[slow] - done[fast] <= delta:
                continue
            fwd = [e[1] for e in sim.order[(slow, s)] if e[0] == "F" and (len(e) == 2 or e[2] == s)]
            if len(fwd) <= 1:
                continue
            for kind in ("stage", "pipeline"):
                offer = (kind, s if kind == "stage" else -1, fwd[-1], slow, fast)
                if offer not in offers:
                    offers.append(offer)
        best = None
        for kind, s, m, slow, fast in offers:
            trial = _move(cur, kind, s, m, slow, fast)
            if trial.assignment == cur.assignment:
                continue
            tsim = simulate(trial, cm, split_backward)
            if tsim.deadlock or not within_caps(tsim):
                continue
            if tsim.makespan < (best[1].makespan if best else sim.makespan) - 1e-12:
                best = (trial, tsim)
        if best is None:
            break
        cur, sim = best
        moves += 1
    return MigrationResult(cur.assignment, sim.makespan, moves, sim, given.makespan)
