"""Progressive TP -> PP -> DP planner producing ``HeteroParallelPlan`` s and IR schedules.

``initial_plan``: place (replica, stage) TP groups (``spread`` by default), partition layers by
min-max DP under memory caps, assign micro-batches, migrate, schedule.

``replan`` after failures / slowdowns, per surviving group of the previous physical plan:
  1. TP: choose a subgroup among the survivors plus free devices of the same node (Eq. 4 over
     every feasible degree -- not only powers of two -- with a memory-derived minimum degree,
     incumbents preferred);
  2. fill missing groups from the free pool (rejoined / spare nodes) and optionally grow
     whole replicas up to ``max_replicas``;
  3. PP: repartition layers by aggregated stage capacity (min-max DP);
  4. DP: progress-aware micro-batch migration (simulated moves);
  5. joint keep-or-evict: for each weakened group, also try dropping it and letting peer
     replicas absorb its work; keep whichever the simulator predicts faster.
Ablation switches ``enable_tp_shrink`` / ``enable_repartition`` / ``enable_migration`` turn
steps off.  (Reference: ``resihp/plan/planner.py:24-273``, ResiHP section 6.)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

from .cost_model import CostModel, Workload
from .dp_migration import initial_assignment, progress_aware_migration, simulate
from .hetero_plan import HeteroParallelPlan, StageGroup, interleave
from .ir import Schedule, compute_order_to_ir, validate
from .layer_partition import counts_to_ranges, partition_layers
from .model_spec import ModelProfile, ModelSpec
from .placement import place_groups
from .simulator import SimResult
from .topology import ClusterTopology
from .tp_select import feasible_degrees, max_layers_for_memory, min_tp_for_memory, select_subgroup

Key = tuple[int, int]


class PlanInfeasible(RuntimeError):
    pass


@dataclass
class PlannerConfig:
    model: ModelSpec
    profile: ModelProfile
    num_stages: int
    num_replicas: int
    tp: int
    num_microbatches: int
    mem_capacity: float = math.inf
    dp_shard: int = 1
    power_of_two_only: bool = False
    sequence_parallel: bool = True
    split_backward: bool = False
    migration_rounds: int = 32
    delta: float = 0.0
    placement: str = "spread"
    workload: Workload | None = None
    enable_tp_shrink: bool = True
    enable_repartition: bool = True
    enable_migration: bool = True
    max_replicas: int | None = None
    vpp: int = 1
    cp: int = 1


class HeteroPlanner:
    def __init__(self, cfg: PlannerConfig):
        self.cfg = cfg

    # ------------------------------------------------------------------ model helpers
    def workload(self) -> Workload:
        c = self.cfg
        return c.workload or Workload.uniform(c.num_microbatches, c.model.seq_len, c.model.micro_batch_size)

    def _extra_params(self, s: int) -> int:
        emb = self.cfg.model.embedding_params()
        return (emb if s == 0 else 0) + (emb if s == self.cfg.num_stages - 1 else 0)

    def _inflight(self, s: int) -> int:
        """In-flight micro-batches at stage ``s`` for memory sizing (CP splits each one)."""
        P, v = self.cfg.num_stages, self.cfg.vpp
        n = max(1, P - s) if v == 1 else math.ceil(((P - s - 1) * 2 + (v - 1) * P) / v) + 1
        return max(1, math.ceil(n / self.cfg.cp))

    def _group_speed(self, devices, speed: dict[str, float]) -> float:
        c = self.cfg
        return c.profile.group_speed(len(devices) // c.cp, min(speed.get(d, 1.0) for d in devices)) * c.cp

    def _k_min(self, layers: int, stage: int) -> int:
        c = self.cfg
        k = min_tp_for_memory(c.model, layers, c.mem_capacity, self._inflight(stage), dp_shard=c.dp_shard,
                              sequence_parallel=c.sequence_parallel, extra_params=self._extra_params(stage))
        return k if k is not None else c.tp + 1  # nothing fits: make every degree infeasible

    def _max_layers(self, tp: int, stage: int) -> int:
        c = self.cfg
        return max_layers_for_memory(c.model, tp, c.mem_capacity, self._inflight(stage), dp_shard=c.dp_shard,
                                     sequence_parallel=c.sequence_parallel, extra_params=self._extra_params(stage))

    def _choose(self, cands: list[tuple[str, float]], max_tp: int, k_min: int, incumbents=None):
        c = self.cfg
        degrees = feasible_degrees(c.model, min(len(cands) // c.cp, max_tp), k_min, c.power_of_two_only)
        return select_subgroup(cands, degrees, c.profile, incumbents=incumbents, cp=c.cp)

    def cost_model(self, plan: HeteroParallelPlan, topology: ClusterTopology) -> CostModel:
        return CostModel(plan, self.cfg.model, self.cfg.profile, self.workload(),
                         {d.id: d.speed for d in topology.devices}, {d.id: d.node for d in topology.devices},
                         split_backward=self.cfg.split_backward)

    def mem_caps(self, plan: HeteroParallelPlan) -> dict[Key, float]:
        """Per physical slot: how many micro-batches' activations fit next to the static state."""
        c = self.cfg
        if math.isinf(c.mem_capacity):
            return {}
        static: dict[Key, float] = {}
        act: dict[Key, float] = {}
        last = plan.num_stages - 1
        emb = c.model.embedding_params()
        for g in plan.stage_groups:
            k = plan.physical_key(g.replica, g.stage)
            extra = (emb if g.stage == 0 else 0) + (emb if g.stage == last else 0)
            static[k] = static.get(k, 0.0) + c.model.static_bytes(g.num_layers, g.tp, c.dp_shard, extra)
            act[k] = act.get(k, 0.0) + c.model.activation_bytes(g.num_layers, g.tp, c.sequence_parallel) / g.cp
        return {k: (math.floor((c.mem_capacity - static[k]) / act[k]) if act[k] > 0 else math.inf) for k in static}

    def _partition(self, capacities: list[float], max_layers: list[int]) -> list[int]:
        c = self.cfg
        if not c.enable_repartition:
            q, r = divmod(c.model.num_layers, c.num_stages)
            return [q + (1 if s < r else 0) for s in range(c.num_stages)]
        return partition_layers(c.model.num_layers, capacities, first_extra=c.profile.first_stage_extra_layers,
                                last_extra=c.profile.last_stage_extra_layers, max_layers=max_layers,
                                min_layers=c.vpp)

    # ------------------------------------------------------------------ plan assembly
    def _assemble(self, generation: int, members: dict[Key, tuple[str, ...]], counts: list[int],
                  world_order: list[str], standby: list[str], topology: ClusterTopology) -> HeteroParallelPlan:
        c = self.cfg
        used = {d for devs in members.values() for d in devs}
        world = [d for d in world_order if d in used] + sorted(used - set(world_order))
        rank = {d: i for i, d in enumerate(world)}
        ranges = counts_to_ranges(counts)
        groups = tuple(StageGroup(r, s, tuple(sorted(devs, key=rank.__getitem__)), ranges[s], c.cp)
                       for (r, s), devs in sorted(members.items(), key=lambda kv: (kv[0][1], kv[0][0])))
        speed = {d.id: d.speed for d in topology.devices}
        assignment = initial_assignment(list(groups), c.num_stages, c.num_microbatches,
                                        lambda key: self._group_speed(members[key], speed))
        plan = HeteroParallelPlan(generation=generation, world=tuple(world), num_layers=c.model.num_layers,
                                  num_stages=c.num_stages, num_replicas=max(r for r, _ in members) + 1,
                                  stage_groups=groups, num_microbatches=c.num_microbatches, assignment=assignment,
                                  standby=tuple(sorted(standby)), sequence_parallel=c.sequence_parallel)
        plan = interleave(plan, c.vpp)
        plan.validate()
        cm = self.cost_model(plan, topology)
        if c.enable_migration:
            res = progress_aware_migration(plan, cm, mem_cap=self.mem_caps(plan) or None, delta=c.delta,
                                           max_rounds=c.migration_rounds, split_backward=c.split_backward)
            plan = replace(plan, assignment=res.assignment)
            makespan, initial = res.makespan, res.initial_makespan
        else:
            makespan = initial = simulate(plan, cm, c.split_backward).makespan
        plan = replace(plan, meta={"predicted_iteration_s": makespan, "unmigrated_iteration_s": initial,
                                   "layer_counts": list(counts)})
        plan.validate()
        return plan

    # ------------------------------------------------------------------ entry points
    def initial_plan(self, topology: ClusterTopology, generation: int = 1) -> HeteroParallelPlan:
        c = self.cfg
        members = place_groups(topology, c.num_replicas, c.num_stages, c.tp * c.cp, c.placement)
        caps = [c.num_replicas * c.profile.group_speed(c.tp, 1.0) * c.cp] * c.num_stages
        counts = self._partition(caps, [self._max_layers(c.tp, s) for s in range(c.num_stages)])
        used = {d for devs in members.values() for d in devs}
        standby = [d for d in topology.ids() if d not in used]
        return self._assemble(generation, members, counts, topology.ids(), standby, topology)

    def replan(self, prev: HeteroParallelPlan, topology: ClusterTopology,
               generation: int | None = None) -> HeteroParallelPlan:
        c = self.cfg
        prev = prev.physical()
        alive = topology.by_id()
        node_of = {d.id: d.node for d in topology.devices}
        grouped = {d for g in prev.stage_groups for d in g.devices}
        pool: dict[str, list[str]] = {}
        for d in topology.devices:
            if d.id in prev.standby or d.id not in grouped:
                pool.setdefault(d.node, []).append(d.id)
        prev_counts = [b - a for a, b in prev.layer_partition()]
        members: dict[Key, tuple[str, ...]] = {}
        for g in sorted(prev.stage_groups, key=lambda g: (g.stage, g.replica)):
            survivors = [d for d in g.devices if d in alive]
            if survivors:
                node = sorted({node_of[d] for d in survivors})[0]
            else:  # the whole group is gone: rebuild on the node with the most free devices
                node = max((n for n in pool if pool[n]), key=lambda n: (len(pool[n]), n), default=None)
            local_free = pool.get(node, []) if node else []
            cands = [(d, alive[d].speed) for d in survivors + local_free]
            if not cands:
                continue
            if not c.enable_tp_shrink:
                if len(survivors) == len(g.devices):
                    members[(g.replica, g.stage)] = tuple(survivors)
                continue
            choice = self._choose(cands, c.tp, self._k_min(prev_counts[g.stage], g.stage),
                                  incumbents=set(survivors))
            if choice is None:
                continue
            members[(g.replica, g.stage)] = choice.devices
            if node:
                pool[node] = [d for d in pool.get(node, []) + survivors if d not in choice.devices]
        self._fill_from_pool(members, pool, alive, prev_counts)
        for s in range(c.num_stages):
            if not any(k[1] == s for k in members):
                raise PlanInfeasible(f"no TP group can host stage {s}")
        gen = prev.generation + 1 if generation is None else generation
        best = self._plan_from_members(members, prev, topology, gen)
        # joint keep-or-evict: Eq. 4 alone cannot see that a weakened group may slow the whole
        # stage more than handing its micro-batches to peer replicas would
        weakened = [k for k, devs in members.items()
                    if len(devs) < c.tp * c.cp or min(alive[d].speed for d in devs) < 1.0]
        for key in weakened:
            if sum(1 for k in members if k[1] == key[1]) < 2:
                continue
            variant = {k: v for k, v in members.items() if k != key}
            try:
                cand = self._plan_from_members(variant, prev, topology, gen)
            except ValueError:
                continue
            if cand.meta["predicted_iteration_s"] < best.meta["predicted_iteration_s"] - 1e-12:
                best = cand
        return best

    def _fill_from_pool(self, members: dict[Key, tuple[str, ...]], pool: dict[str, list[str]], alive: dict,
                        prev_counts: list[int]) -> None:
        """Rejoin / grow: rebuild missing (replica, stage) groups of the nominal layout from free
        devices, then add whole replicas up to ``max_replicas``."""
        c = self.cfg
        target = max(c.num_replicas, c.max_replicas or 0)
        slot = c.tp * c.cp

        def take(stage: int) -> tuple[str, ...] | None:
            for node in sorted(pool, key=lambda n: (-len(pool[n]), n)):
                cands = [(d, alive[d].speed) for d in pool[node]]
                if not cands:
                    continue
                choice = self._choose(cands, c.tp, self._k_min(prev_counts[stage], stage))
                if choice is not None and choice.tp == c.tp:
                    pool[node] = [d for d in pool[node] if d not in choice.devices]
                    return choice.devices
            return None

        for r in range(target):
            missing = [s for s in range(c.num_stages) if (r, s) not in members]
            if not missing:
                continue
            if r >= c.num_replicas:
                if len(missing) < c.num_stages:
                    continue
                if sum(len(v) // slot for v in pool.values()) < c.num_stages:
                    break
            for s in missing:
                devs = take(s)
                if devs is not None:
                    members[(r, s)] = devs

    def _plan_from_members(self, members: dict[Key, tuple[str, ...]], prev: HeteroParallelPlan,
                           topology: ClusterTopology, gen: int) -> HeteroParallelPlan:
        c = self.cfg
        alive = topology.by_id()
        speed = {d: alive[d].speed for devs in members.values() for d in devs}
        caps, max_layers = [], []
        for s in range(c.num_stages):
            keys = [k for k in members if k[1] == s]
            caps.append(sum(self._group_speed(members[k], speed) for k in keys))
            max_layers.append(min(self._max_layers(len(members[k]) // c.cp, s) for k in keys))
        counts = self._partition(caps, max_layers)
        used = {d for devs in members.values() for d in devs}
        standby = [d for d in topology.ids() if d not in used]
        return self._assemble(gen, members, counts, list(prev.world), standby, topology)

    def schedule(self, plan: HeteroParallelPlan, topology: ClusterTopology) -> tuple[Schedule, SimResult]:
        sim = simulate(plan, self.cost_model(plan, topology), self.cfg.split_backward)
        ir = compute_order_to_ir(plan, sim.order)
        validate(plan, ir, self.cfg.split_backward)
        return ir, sim
