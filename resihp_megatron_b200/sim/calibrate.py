"""Fits the cluster simulator's ResiHP throughput model to the real planner.

At a scale where planning is cheap (TP8 x PP4 x DP 2/4/8) the planner and its pipeline
simulator predict the degraded iteration time of three canonical degradations: one GPU lost,
one whole TP group lost, one GPU running 2x slow.  The analytic model of ``sim.cluster`` has two
free parameters, the repartition blend ``beta`` and the overhead factor; fitting them jointly
over several DP sizes separates the ``1/D`` (bottleneck) and ``1/(S D)`` (repartitioned) scaling
of the deficit, which is what extrapolating to 1K-64K GPUs needs.
Parity: ``resihp/sim/calibrate.py:25-76`` (same scenarios, grid and fit).
"""

from __future__ import annotations

import itertools
import math

from ..plan.model_spec import ModelProfile, ModelSpec
from ..plan.planner import HeteroPlanner, PlannerConfig
from ..plan.topology import ClusterTopology
from ..plan.tp_select import feasible_degrees
from .cluster import ClusterState, JobConfig, resihp_params

MODEL = ModelSpec(num_layers=40, hidden=5120, ffn=13824, num_heads=40, num_kv_heads=40, vocab=32000, seq_len=4096)
PROFILE = ModelProfile(alpha=3.0e-6, beta=1.0e-10)
MB_PER_REPLICA = 16
SCENARIOS = ("lose_gpu", "lose_group", "slow_gpu_2x")
BETAS = [b / 20 for b in range(21)]            # 0.00 .. 1.00
OVERHEADS = [o / 20 for o in range(5, 61)]     # 0.25 .. 3.00


def measured(tp: int = 8, pp: int = 4, dp: int = 4, microbatches: int = 32) -> dict[str, float]:
    """Relative throughput (healthy / degraded predicted iteration time) according to the planner."""
    planner = HeteroPlanner(PlannerConfig(model=MODEL, profile=PROFILE, num_stages=pp, num_replicas=dp, tp=tp,
                                          num_microbatches=microbatches, mem_capacity=80e9, migration_rounds=24))
    topo = ClusterTopology.uniform(tp * pp * dp // 8, 8, nodes_per_rack=2)
    plan = planner.initial_plan(topo)
    victims = plan.group(0, 1).devices
    variants = {"lose_gpu": topo.without({victims[0]}), "lose_group": topo.without(set(victims)),
                "slow_gpu_2x": topo.with_speeds({victims[0]: 0.5})}
    healthy = plan.meta["predicted_iteration_s"]
    return {name: healthy / planner.replan(plan, t).meta["predicted_iteration_s"] for name, t in variants.items()}


def _degrade(st: ClusterState, scenario: str, group: list[int]) -> None:
    if scenario == "lose_gpu":
        st.lost[group[0]] = math.inf
    elif scenario == "lose_group":
        st.lost.update((g, math.inf) for g in group)
    else:
        st.slow[group[0]] = (2.0, math.inf, True)


def modelled(job: JobConfig, beta: float, overhead: float) -> dict[str, float]:
    """The simulator model's relative throughput in each scenario."""
    policy = resihp_params(job, beta=beta, overhead=overhead)
    group = list(job.group_gpus(0, 1))
    result = {}
    for scenario in SCENARIOS:
        st = ClusterState(job, policy)
        _degrade(st, scenario, group)
        st.refresh(group)
        result[scenario] = st.throughput()
    return result


def calibrate(tp: int = 8, pp: int = 4, dps: tuple[int, ...] = (2, 4, 8)) -> dict:
    degrees = tuple(feasible_degrees(MODEL, tp))
    truth = {dp: measured(tp, pp, dp, microbatches=MB_PER_REPLICA * dp) for dp in dps}
    jobs = {dp: JobConfig(gpus=tp * pp * dp, tp=tp, pp=pp, min_tp=1, tp_degrees=degrees, profile=PROFILE,
                          microbatches_per_replica=MB_PER_REPLICA) for dp in dps}

    def sse(beta: float, overhead: float):
        preds = {dp: modelled(jobs[dp], beta, overhead) for dp in dps}
        return sum((preds[dp][k] - truth[dp][k]) ** 2 for dp in dps for k in SCENARIOS), preds

    best = None
    for beta, overhead in itertools.product(BETAS, OVERHEADS):
        err, preds = sse(beta, overhead)
        if best is None or err < best[0] - 1e-15:  # ties keep the earlier grid point
            best = (err, beta, overhead, preds)
    err, beta, overhead, preds = best
    return {"beta": beta, "overhead": overhead, "rmse": math.sqrt(err / (len(dps) * len(SCENARIOS))),
            "measured": {str(dp): m for dp, m in truth.items()}, "model": {str(dp): p for dp, p in preds.items()},
            "scale": {"tp": tp, "pp": pp, "dp": list(dps)}, "tp_degrees": list(degrees)}
