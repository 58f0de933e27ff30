"""The joint TP -> PP -> DP planner: produces ``HeteroParallelPlan`` s and their IR schedules.

``initial_plan``: place the (replica, stage) TP groups (``spread`` by default), split the layers
by the min-max partition under the memory caps, assign micro-batches, migrate, schedule.

``replan`` after failures or slowdowns works from the previous physical plan, group by group:

1. **TP** -- for each group pick a subgroup among its survivors and the free devices of its
   node: Eq. 4 over every feasible degree (not only powers of two), no smaller than the degree
   the stage's memory needs, incumbents first.  A group with no survivor is rebuilt on the node
   with the most free devices.
2. **Pool** -- rebuild missing groups of the nominal layout from free devices (rejoined or spare
   nodes), and optionally grow whole replicas up to ``max_replicas``.
3. **PP** -- repartition the layers by each stage's aggregate capacity.
4. **DP** -- progress-aware micro-batch migration, every move checked by simulation.
5. **Keep or evict** -- for every weakened group (fewer devices or a slow member) also try
   dropping it and letting its stage's other replicas absorb its work; keep the faster plan.

``enable_tp_shrink`` / ``enable_repartition`` / ``enable_migration`` switch steps off for the
ablation study.  Parity: ``resihp/plan/planner.py:24-273`` (ResiHP section 6; same steps and
config fields).
"""

from __future__ import annotations

import math
from collections import defaultdict
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


class _Memory:
    """The per-GPU memory model of one stage under a config."""

    def __init__(self, cfg: PlannerConfig):
        self.cfg = cfg

    def extra_params(self, stage: int) -> int:
        emb = self.cfg.model.embedding_params()
        return emb * ((stage == 0) + (stage == self.cfg.num_stages - 1))

    def inflight(self, stage: int) -> int:
        """Micro-batches stage ``stage`` holds at once (1F1B or interleaved warm-up), CP-split."""
        P, v = self.cfg.num_stages, self.cfg.vpp
        depth = max(1, P - stage) if v == 1 else math.ceil(((P - stage - 1) * 2 + (v - 1) * P) / v) + 1
        return max(1, math.ceil(depth / self.cfg.cp))

    def _kw(self, stage: int) -> dict:
        return dict(dp_shard=self.cfg.dp_shard, sequence_parallel=self.cfg.sequence_parallel,
                    extra_params=self.extra_params(stage))

    def min_tp(self, layers: int, stage: int) -> int:
        k = min_tp_for_memory(self.cfg.model, layers, self.cfg.mem_capacity, self.inflight(stage), **self._kw(stage))
        return self.cfg.tp + 1 if k is None else k  # nothing fits: no degree is allowed

    def max_layers(self, tp: int, stage: int) -> int:
        return max_layers_for_memory(self.cfg.model, tp, self.cfg.mem_capacity, self.inflight(stage),
                                     **self._kw(stage))

    def slot_caps(self, plan: HeteroParallelPlan) -> dict[Key, float]:
        """Per physical slot: how many micro-batches' activations fit beside its static state."""
        c = self.cfg
        if math.isinf(c.mem_capacity):
            return {}
        static, per_mb = defaultdict(float), defaultdict(float)
        for g in plan.stage_groups:
            slot = plan.physical_key(g.replica, g.stage)
            static[slot] += c.model.static_bytes(g.num_layers, g.tp, c.dp_shard, self.extra_params(g.stage))
            per_mb[slot] += c.model.activation_bytes(g.num_layers, g.tp, c.sequence_parallel) / g.cp
        return {k: math.floor((c.mem_capacity - static[k]) / per_mb[k]) if per_mb[k] > 0 else math.inf
                for k in static}


class HeteroPlanner:
    def __init__(self, cfg: PlannerConfig):
        self.cfg = cfg
        self.mem = _Memory(cfg)

    # ------------------------------------------------------------------ pricing
    def workload(self) -> Workload:
        c = self.cfg
        return c.workload or Workload.uniform(c.num_microbatches, c.model.seq_len, c.model.micro_batch_size)

    def cost_model(self, plan: HeteroParallelPlan, topology: ClusterTopology) -> CostModel:
        speeds = {d.id: d.speed for d in topology.devices}
        nodes = {d.id: d.node for d in topology.devices}
        return CostModel(plan, self.cfg.model, self.cfg.profile, self.workload(), speeds, nodes,
                         split_backward=self.cfg.split_backward)

    def mem_caps(self, plan: HeteroParallelPlan) -> dict[Key, float]:
        return self.mem.slot_caps(plan)

    def _speed_of(self, devices, speed: dict[str, float]) -> float:
        c = self.cfg
        return c.cp * c.profile.group_speed(len(devices) // c.cp, min(speed.get(d, 1.0) for d in devices))

    def _subgroup(self, candidates, k_min: int, incumbents=None):
        c = self.cfg
        top = min(len(candidates) // c.cp, c.tp)
        degrees = feasible_degrees(c.model, top, k_min, c.power_of_two_only)
        return select_subgroup(candidates, degrees, c.profile, incumbents=incumbents, cp=c.cp)

    def _layer_counts(self, capacities: list[float], max_layers: list[int]) -> list[int]:
        c = self.cfg
        if c.enable_repartition:
            return partition_layers(c.model.num_layers, capacities, first_extra=c.profile.first_stage_extra_layers,
                                    last_extra=c.profile.last_stage_extra_layers, max_layers=max_layers,
                                    min_layers=c.vpp)
        base, rest = divmod(c.model.num_layers, c.num_stages)
        return [base + int(s < rest) for s in range(c.num_stages)]

    # ------------------------------------------------------------------ assembly
    def _build(self, generation: int, members: dict[Key, tuple[str, ...]], counts: list[int],
               world_order: list[str], topology: ClusterTopology) -> HeteroParallelPlan:
        c = self.cfg
        used = {d for devs in members.values() for d in devs}
        world = [d for d in world_order if d in used]
        world += sorted(used.difference(world_order))
        pos = {d: i for i, d in enumerate(world)}
        spans = counts_to_ranges(counts)
        groups = tuple(StageGroup(r, s, tuple(sorted(members[(r, s)], key=pos.__getitem__)), spans[s], c.cp)
                       for r, s in sorted(members, key=lambda k: (k[1], k[0])))
        speed = {d.id: d.speed for d in topology.devices}
        table = initial_assignment(list(groups), c.num_stages, c.num_microbatches,
                                   lambda key: self._speed_of(members[key], speed))
        plan = HeteroParallelPlan(generation=generation, world=tuple(world), num_layers=c.model.num_layers,
                                  num_stages=c.num_stages, num_replicas=1 + max(r for r, _ in members),
                                  stage_groups=groups, num_microbatches=c.num_microbatches, assignment=table,
                                  standby=tuple(sorted(d for d in topology.ids() if d not in used)),
                                  sequence_parallel=c.sequence_parallel)
        plan = interleave(plan, c.vpp)
        plan.validate()
        cm = self.cost_model(plan, topology)
        if c.enable_migration:
            moved = progress_aware_migration(plan, cm, mem_cap=self.mem_caps(plan) or None, delta=c.delta,
                                             max_rounds=c.migration_rounds, split_backward=c.split_backward)
            plan = replace(plan, assignment=moved.assignment)
            predicted, before = moved.makespan, moved.initial_makespan
        else:
            predicted = before = simulate(plan, cm, c.split_backward).makespan
        plan = replace(plan, meta={"predicted_iteration_s": predicted, "unmigrated_iteration_s": before,
                                   "layer_counts": list(counts)})
        plan.validate()
        return plan

    def _from_members(self, members: dict[Key, tuple[str, ...]], prev: HeteroParallelPlan,
                      topology: ClusterTopology, generation: int) -> HeteroParallelPlan:
        c = self.cfg
        speed = {d.id: d.speed for d in topology.devices}
        capacity, ceiling = [], []
        for s in range(c.num_stages):
            here = [devs for (r, st), devs in members.items() if st == s]
            capacity.append(sum(self._speed_of(devs, speed) for devs in here))
            ceiling.append(min(self.mem.max_layers(len(devs) // c.cp, s) for devs in here))
        return self._build(generation, members, self._layer_counts(capacity, ceiling), list(prev.world), topology)

    # ------------------------------------------------------------------ entry points
    def initial_plan(self, topology: ClusterTopology, generation: int = 1) -> HeteroParallelPlan:
        c = self.cfg
        members = place_groups(topology, c.num_replicas, c.num_stages, c.tp * c.cp, c.placement)
        stage_capacity = c.num_replicas * c.cp * c.profile.group_speed(c.tp, 1.0)
        counts = self._layer_counts([stage_capacity] * c.num_stages,
                                    [self.mem.max_layers(c.tp, s) for s in range(c.num_stages)])
        return self._build(generation, members, counts, topology.ids(), topology)

    def _regroup(self, prev: HeteroParallelPlan, topology: ClusterTopology, counts: list[int]):
        """Step 1: a subgroup per surviving group; returns the members and the free-device pool."""
        c = self.cfg
        alive = topology.by_id()
        grouped = {d for g in prev.stage_groups for d in g.devices}
        pool: dict[str, list[str]] = defaultdict(list)
        for d in topology.devices:
            if d.id in prev.standby or d.id not in grouped:
                pool[d.node].append(d.id)
        members: dict[Key, tuple[str, ...]] = {}
        for g in sorted(prev.stage_groups, key=lambda g: (g.stage, g.replica)):
            survivors = [d for d in g.devices if d in alive]
            if survivors:
                node = min(alive[d].node for d in survivors)
            else:  # the whole group is gone: rebuild it where most devices are free
                roomy = [n for n in pool if pool[n]]
                node = max(roomy, key=lambda n: (len(pool[n]), n)) if roomy else None
            candidates = [(d, alive[d].speed) for d in survivors + (list(pool[node]) if node else [])]
            if not candidates:
                continue
            if not c.enable_tp_shrink:
                if len(survivors) == len(g.devices):
                    members[(g.replica, g.stage)] = tuple(survivors)
                continue
            pick = self._subgroup(candidates, self.mem.min_tp(counts[g.stage], g.stage), incumbents=set(survivors))
            if pick is None:
                continue
            members[(g.replica, g.stage)] = pick.devices
            if node:
                pool[node] = [d for d in pool[node] + survivors if d not in pick.devices]
        return members, pool

    def _fill_from_pool(self, members: dict[Key, tuple[str, ...]], pool: dict[str, list[str]], alive: dict,
                        prev_counts: list[int]) -> None:
        """Step 2: rebuild missing groups of the nominal layout from free devices, then grow whole
        replicas up to ``max_replicas``."""
        c = self.cfg
        width = c.tp * c.cp

        def full_group(stage: int) -> tuple[str, ...] | None:
            for node in sorted(pool, key=lambda n: (-len(pool[n]), n)):
                if not pool[node]:
                    continue
                pick = self._subgroup([(d, alive[d].speed) for d in pool[node]],
                                      self.mem.min_tp(prev_counts[stage], stage))
                if pick is not None and pick.tp == c.tp:
                    pool[node] = [d for d in pool[node] if d not in pick.devices]
                    return pick.devices
            return None

        for r in range(max(c.num_replicas, c.max_replicas or 0)):
            gaps = [s for s in range(c.num_stages) if (r, s) not in members]
            if not gaps:
                continue
            if r >= c.num_replicas:  # growing: only whole new replicas, only if the pool can hold one
                if len(gaps) < c.num_stages:
                    continue
                if sum(len(v) // width for v in pool.values()) < c.num_stages:
                    break
            for s in gaps:
                devs = full_group(s)
                if devs is not None:
                    members[(r, s)] = devs

    def replan(self, prev: HeteroParallelPlan, topology: ClusterTopology,
               generation: int | None = None) -> HeteroParallelPlan:
        c = self.cfg
        prev = prev.physical()
        alive = topology.by_id()
        counts = [hi - lo for lo, hi in prev.layer_partition()]
        members, pool = self._regroup(prev, topology, counts)
        self._fill_from_pool(members, pool, alive, counts)
        orphaned = [s for s in range(c.num_stages) if all(k[1] != s for k in members)]
        if orphaned:
            raise PlanInfeasible(f"no TP group can host stage {orphaned[0]}")
        gen = generation if generation is not None else prev.generation + 1
        best = self._from_members(members, prev, topology, gen)
        # Step 5: Eq. 4 alone cannot see that a weakened group may slow its whole stage more than
        # handing its micro-batches to the stage's other replicas would.
        replicas_at = defaultdict(int)
        for _, s in members:
            replicas_at[s] += 1
        for key, devs in list(members.items()):
            weakened = len(devs) < c.tp * c.cp or min(alive[d].speed for d in devs) < 1.0
            if not weakened or replicas_at[key[1]] < 2:
                continue
            try:
                trial = self._from_members({k: v for k, v in members.items() if k != key}, prev, topology, gen)
            except ValueError:
                continue
            if trial.meta["predicted_iteration_s"] < best.meta["predicted_iteration_s"] - 1e-12:
                best = trial
        return best

    def schedule(self, plan: HeteroParallelPlan, topology: ClusterTopology) -> tuple[Schedule, SimResult]:
        """The simulated order of ``plan`` as a validated IR, with its simulation."""
        sim = simulate(plan, self.cost_model(plan, topology), self.cfg.split_backward)
        ir = compute_order_to_ir(plan, sim.order)
        validate(plan, ir, self.cfg.split_backward)
        return ir, sim
