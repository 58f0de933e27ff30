"""Replica-level planner: whole-replica exclusion (the baseline torchft offers), but with the
global batch preserved by redistributing the lost replica's micro-batches by speed, and with
state sources chosen same-node first.  (Reference: ``resihp/plan/dp_planner.py:11-56``.)
"""

from __future__ import annotations

from ..control.coordinator import ClusterView
from ..state.transaction import roll_forward_plan
from .dp_migration import largest_remainder


def weighted_assignment(workers: list[str], num_microbatches: int, weights: dict[str, float]) -> dict[str, list[int]]:
    """Contiguous micro-batch ranges proportional to speed (largest-remainder rounding)."""
    counts = largest_remainder(num_microbatches, [max(weights.get(w, 1.0), 1e-9) for w in workers])
    out, a = {}, 0
    for w, c in zip(workers, counts):
        out[w] = list(range(a, a + c))
        a += c
    return out


def assign_sources(needs: list[str], providers: list[str], node_of: dict[str, str]) -> dict[str, str]:
    """A provider per receiver: same node first, then the least-loaded provider."""
    if not providers:
        return {}
    load = dict.fromkeys(providers, 0)
    out = {}
    for w in needs:
        local = [p for p in providers if node_of.get(p) == node_of.get(w)]
        src = min(local or providers, key=lambda p: (load[p], providers.index(p)))
        load[src] += 1
        out[w] = src
    return out


def make_dp_planner(num_microbatches: int, min_speed: float = 0.0):
    def planner(view: ClusterView) -> tuple[list[str], dict]:
        alive = view.alive
        world = [w.worker_id for w in alive if w.health.get("p", 1.0) >= min_speed] or [w.worker_id for w in alive]
        weights = {w.worker_id: float(w.health.get("p", 1.0)) for w in alive}
        node_of = {w.worker_id: w.node_id for w in alive}
        rec = roll_forward_plan(view.recovery, world)
        restore = None
        if rec["target_iteration"] >= 0 and not rec["up_to_date"] and not rec["local_step"]:
            restore = "checkpoint"
        rec["sources"] = assign_sources(rec["needs_state"], rec["up_to_date"] + rec["local_step"], node_of)
        rec["restore"] = restore
        payload = {"kind": "dp", "num_microbatches": num_microbatches,
                   "assignment": weighted_assignment(world, num_microbatches, weights), "recovery": rec}
        return world, payload

    return planner
