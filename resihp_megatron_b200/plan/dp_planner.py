"""Replica-level planner: a failed or too-slow replica is dropped as a whole (the recovery that
torchft-style systems offer), but the global batch is preserved -- the micro-batches are dealt
to the remaining workers by speed -- and each worker that needs state gets a source on its own
node when one exists.  It is the coordinator's ``PlannerFn`` for the data-parallel runtime.
Parity: ``resihp/plan/dp_planner.py:11-56`` (same payload: ``kind``, ``num_microbatches``,
``assignment``, ``recovery``).
"""

from __future__ import annotations

import itertools
from collections import Counter

from ..control.coordinator import ClusterView
from ..state.transaction import roll_forward_plan
from .dp_migration import largest_remainder


def weighted_assignment(workers: list[str], num_microbatches: int, weights: dict[str, float]) -> dict[str, list[int]]:
    """Consecutive micro-batch ids per worker, shares proportional to speed."""
    shares = largest_remainder(num_microbatches, [max(weights.get(w, 1.0), 1e-9) for w in workers])
    bounds = list(itertools.accumulate(shares, initial=0))
    return {w: list(range(a, b)) for w, a, b in zip(workers, bounds, bounds[1:])}


def assign_sources(needs: list[str], providers: list[str], node_of: dict[str, str]) -> dict[str, str]:
    """One state provider per receiver: providers on the receiver's node first, then the least
    used so far (earlier in ``providers`` on ties)."""
    rank = {p: i for i, p in enumerate(providers)}
    used: Counter = Counter()
    chosen = {}
    for w in needs:
        pool = [p for p in providers if node_of.get(p) == node_of.get(w)] or providers
        if not pool:
            return {}
        src = min(pool, key=lambda p: (used[p], rank[p]))
        used[src] += 1
        chosen[w] = src
    return chosen


def make_dp_planner(num_microbatches: int, min_speed: float = 0.0):
    """Planner for ``num_microbatches`` per iteration; workers whose reported speed ``p`` is
    below ``min_speed`` are left out (unless that would leave nobody)."""

    def planner(view: ClusterView) -> tuple[list[str], dict]:
        speed = {w.worker_id: float(w.health.get("p", 1.0)) for w in view.alive}
        world = [w for w, p in speed.items() if p >= min_speed] or list(speed)
        recovery = roll_forward_plan(view.recovery, world)
        holders = recovery["up_to_date"] + recovery["local_step"]
        recovery["sources"] = assign_sources(recovery["needs_state"], holders,
                                             {w.worker_id: w.node_id for w in view.alive})
        needs_checkpoint = recovery["target_iteration"] >= 0 and not holders
        recovery["restore"] = "checkpoint" if needs_checkpoint else None
        return world, {"kind": "dp", "num_microbatches": num_microbatches,
                       "assignment": weighted_assignment(world, num_microbatches, speed), "recovery": recovery}

    return planner
