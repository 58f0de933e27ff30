"""Planner ablation: the planner's predicted throughput after canonical degradations
(healthy = 1).

Variants: the full planner; no TP shrink (a weakened group is evicted instead); no layer
repartition; no micro-batch migration; and whole-replica exclusion with the global batch kept
(torchft-style replica drop).
Parity: ``resihp/bench/planner_ablation.py:1-61`` (same variants, scenarios and table).
"""

from __future__ import annotations

from dataclasses import replace

from ..plan.planner import HeteroPlanner, PlanInfeasible, PlannerConfig
from ..plan.topology import ClusterTopology
from ..sim.calibrate import MODEL, PROFILE

VARIANTS = {"ResiHP": {}, "no TP shrink": {"enable_tp_shrink": False},
            "no repartition": {"enable_repartition": False}, "no migration": {"enable_migration": False}}
SLOW_REPLICA_DROP = 0.5  # synchronous DP waits for the 2x slow replica


def _speedup(planner: HeteroPlanner, plan, topo, healthy_s: float) -> float | None:
    """Healthy / replanned predicted iteration time; None when no plan exists ("stops")."""
    try:
        return healthy_s / planner.replan(plan, topo).meta["predicted_iteration_s"]
    except PlanInfeasible:
        return None


def _scenarios(plan, topo) -> dict:
    victim = plan.group(0, 1).devices
    return {"1 GPU lost": topo.without({victim[0]}),
            "2 GPUs lost (2 replicas)": topo.without({victim[0], plan.group(1, 1).devices[0]}),
            "node lost": topo.without(set(victim)),
            "1 GPU 2x slow": topo.with_speeds({victim[0]: 0.5})}


def run(dps=(2, 4), tp: int = 8, pp: int = 4, mb_per_replica: int = 16) -> list[dict]:
    rows = []
    for dp in dps:
        cfg = PlannerConfig(model=MODEL, profile=PROFILE, num_stages=pp, num_replicas=dp, tp=tp,
                            num_microbatches=mb_per_replica * dp, mem_capacity=80e9, migration_rounds=32)
        topo = ClusterTopology.uniform(tp * pp * dp // 8, 8, nodes_per_rack=2)
        plan = HeteroPlanner(cfg).initial_plan(topo)
        healthy_s = plan.meta["predicted_iteration_s"]
        first_replica = {d for g in plan.stage_groups if g.replica == 0 for d in g.devices}
        for name, degraded in _scenarios(plan, topo).items():
            row = {"gpus": tp * pp * dp, "dp": dp, "scenario": name}
            row.update((variant, _speedup(HeteroPlanner(replace(cfg, **kw)), plan, degraded, healthy_s))
                       for variant, kw in VARIANTS.items())
            if name == "1 GPU 2x slow":
                row["replica drop"] = SLOW_REPLICA_DROP
            else:
                gone = set(topo.ids()) - set(degraded.ids())
                row["replica drop"] = _speedup(HeteroPlanner(cfg), plan, topo.without(first_replica | gone), healthy_s)
            rows.append(row)
    return rows


def to_markdown(rows: list[dict]) -> str:
    columns = [*VARIANTS, "replica drop"]

    def cell(value) -> str:
        return "stops" if value is None else f"{value:.3f}"

    table = ["| GPUs | scenario | " + " | ".join(columns) + " |", "|---|---|" + "---|" * len(columns)]
    table += [f"| {r['gpus']} | {r['scenario']} | " + " | ".join(cell(r[c]) for c in columns) + " |" for r in rows]
    table.append(f"\n`replica drop` for a slow GPU: synchronous DP waits for the slow replica "
                 f"({SLOW_REPLICA_DROP} at 2x).")
    return "\n".join(table)
