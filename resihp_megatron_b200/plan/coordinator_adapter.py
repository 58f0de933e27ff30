"""Connects the coordinator's planner callback to the heterogeneous planner.

The coordinator calls ``planner(view) -> (world, payload)`` inside every reconfiguration
transaction.  The payload it broadcasts in PREPARE carries everything a worker needs to enter
the new generation without talking to anyone else: the new plan, its validated IR schedule,
the previous plan (each worker derives the same slice-transfer plan from the pair), the
roll-forward recovery decision and the device -> node map.  Plans for single-device losses
are precomputed in the background (``PlanCache``) and taken from there when the cluster is
otherwise healthy.  When the survivors cannot keep every pipeline stage alive at the current
replica count, the job is rebuilt with fewer replicas and state is restored from snapshots or
checkpoints.  ``make_what_if`` prices a confirmed slowdown for the ski-rental policy.
(Reference: ``resihp/plan/coordinator_adapter.py:27-111``.)
"""

from __future__ import annotations

import time
from dataclasses import dataclass, replace

from ..state.transaction import roll_forward_plan
from ..utils.log import get_logger
from .hetero_plan import HeteroParallelPlan
from .ir import schedule_to_json
from .plan_cache import PlanCache
from .planner import HeteroPlanner, PlanInfeasible, PlannerConfig
from .reconfig_cost import estimate_reconfig_cost, gpt_layer_specs
from .topology import ClusterTopology, Device

log = get_logger(__name__)


def topology_from_view(view) -> ClusterTopology:
    """Alive workers as planner devices; ``health['p']`` is the relative speed, ``health['rack']``
    the failure domain."""
    return ClusterTopology(tuple(
        Device(w.worker_id, w.node_id, w.local_rank, str(w.health.get("rack", "r0")), float(w.health.get("p", 1.0)))
        for w in view.alive))


def topology_from_nodes(nodes: dict[str, str], speeds: dict[str, float] | None = None) -> ClusterTopology:
    speeds = speeds or {}
    rank_in_node: dict[str, int] = {}
    devices = []
    for dev, node in nodes.items():
        devices.append(Device(dev, node, rank_in_node.get(node, 0), "r0", float(speeds.get(dev, 1.0))))
        rank_in_node[node] = rank_in_node.get(node, 0) + 1
    return ClusterTopology(tuple(devices))


class HeteroPlannerFn:
    """The coordinator-facing planner.  ``cache`` is exposed for inspection and tests."""

    def __init__(self, cfg: PlannerConfig, use_cache: bool = True):
        self.cfg = cfg
        self.planner = HeteroPlanner(cfg)
        self.cache = PlanCache(lambda p, t: self.planner.replan(p, t)) if use_cache else None

    def _previous(self, view) -> HeteroParallelPlan | None:
        prev = view.previous_payload
        if prev and prev.get("kind") == "hetero":
            return HeteroParallelPlan.from_json(prev["plan"])
        return None

    def _from_cache(self, prev: HeteroParallelPlan, topo: ClusterTopology, view) -> HeteroParallelPlan | None:
        if self.cache is None:
            return None
        failed = set(prev.world) - set(topo.ids())
        if not failed or any(float(w.health.get("p", 1.0)) < 1.0 for w in view.alive):
            return None  # cached plans assume full-speed survivors
        hit = self.cache.lookup(prev.generation, set(topo.ids()), failed)
        return replace(hit, generation=view.generation) if hit is not None else None

    def _shrunk_initial(self, topo: ClusterTopology, generation: int) -> HeteroParallelPlan:
        slots = sum(len(devs) // self.cfg.tp for devs in topo.nodes().values())
        replicas = max(1, slots // self.cfg.num_stages)
        return HeteroPlanner(replace(self.cfg, num_replicas=replicas)).initial_plan(topo, generation=generation)

    def _degraded_initial(self, topo: ClusterTopology, generation: int) -> HeteroParallelPlan:
        """A job that starts with fewer devices than its nominal layout (a node short of a GPU):
        plan the nominal layout on a topology padded with placeholder devices, then re-plan
        without them, exactly as if they had failed (TP shrink, repartition, migration)."""
        from .topology import Device

        nodes = topo.nodes()
        width = max(len(d) for d in nodes.values())
        width = -(-width // self.cfg.tp) * self.cfg.tp
        devs = list(topo.devices)
        for node, have in nodes.items():
            for k in range(len(have), width):
                devs.append(Device(f"{node}~{k}", node, k, have[0].rack))
        padded = ClusterTopology(tuple(devs))
        nominal = self.planner.initial_plan(padded, generation=generation)
        return self.planner.replan(nominal, topo, generation=generation)

    def __call__(self, view) -> tuple[list[str], dict]:
        t0 = time.monotonic()
        topo = topology_from_view(view)
        prev = self._previous(view)
        restore = None
        hit = False
        if prev is None:
            try:
                plan = self.planner.initial_plan(topo, generation=view.generation)
            except (ValueError, PlanInfeasible):
                plan = self._degraded_initial(topo, view.generation)
        else:
            plan = self._from_cache(prev, topo, view)
            hit = plan is not None
            if plan is None:
                try:
                    plan = self.planner.replan(prev, topo, generation=view.generation)
                except PlanInfeasible as e:
                    log.error("replan infeasible (%s): rebuilding with fewer replicas from saved state", e)
                    plan = self._shrunk_initial(topo, view.generation)
                    restore = "snapshot_or_checkpoint"
        schedule, sim = self.planner.schedule(plan, topo)
        world = list(plan.world)
        recovery = roll_forward_plan(view.recovery, world)
        recovery["restore"] = restore
        payload = {
            "kind": "hetero",
            "plan": plan.to_json(),
            "schedule": schedule_to_json(schedule),
            "previous_plan": prev.to_json() if prev is not None else None,
            "recovery": recovery,
            "predicted_iteration_s": sim.makespan,
            "nodes": {d.id: d.node for d in topo.devices},
            "planning_s": time.monotonic() - t0,
            "plan_cache_hit": hit,
        }
        if self.cache is not None:
            self.cache.warm(plan, topo)
        return world, payload


def make_hetero_planner(cfg: PlannerConfig, use_cache: bool = True) -> HeteroPlannerFn:
    return HeteroPlannerFn(cfg, use_cache)


@dataclass(frozen=True)
class WhatIf:
    current_s: float     # predicted iteration time if the committed plan is kept
    mitigated_s: float   # predicted iteration time after replanning around the slow devices
    reconfig_s: float    # one-off reconfiguration cost
    bytes_moved: int


def make_what_if(cfg: PlannerConfig, **cost_kw):
    """``what_if(payload, speeds) -> WhatIf`` for the committed generation's payload.  Times are
    in the profile's units: calibrate the profile to seconds before comparing with wall clock."""
    planner = HeteroPlanner(cfg)
    specs = gpt_layer_specs(cfg.model)

    def what_if(payload: dict, speeds: dict[str, float]) -> WhatIf:
        prev = HeteroParallelPlan.from_json(payload["plan"])
        nodes: dict[str, str] = payload["nodes"]
        topo = topology_from_nodes(nodes, speeds)
        _, sim = planner.schedule(prev, topo)
        new = planner.replan(prev, topo)
        est = estimate_reconfig_cost(prev, new, specs, node_of=nodes, **cost_kw)
        return WhatIf(sim.makespan, new.meta["predicted_iteration_s"], est.seconds, est.bytes_moved)

    return what_if
