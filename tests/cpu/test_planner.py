"""Planner behaviour after failures and slowdowns, its ablations, plan cache, reconfiguration
cost, rejoin / grow, and the coordinator adapter."""

import time
from dataclasses import replace

import pytest

from resihp_megatron_b200.plan.model_spec import ModelProfile, ModelSpec
from resihp_megatron_b200.plan.plan_cache import PlanCache
from resihp_megatron_b200.plan.planner import HeteroPlanner, PlanInfeasible, PlannerConfig
from resihp_megatron_b200.plan.reconfig_cost import estimate_reconfig_cost, gpt_layer_specs
from resihp_megatron_b200.plan.topology import ClusterTopology

LLAMA13B = ModelSpec(num_layers=40, hidden=5120, ffn=13824, num_heads=40, num_kv_heads=40, vocab=32000, seq_len=4096)
PROFILE = ModelProfile(alpha=3.0e-6, beta=1.0e-10, last_stage_extra_layers=1.0)


def planner(**kw):
    cfg = PlannerConfig(model=LLAMA13B, profile=PROFILE, num_stages=4, num_replicas=2, tp=4, num_microbatches=16,
                        mem_capacity=80e9, migration_rounds=48)
    return HeteroPlanner(replace(cfg, **kw))


def topo():
    return ClusterTopology.uniform(4, 8, nodes_per_rack=2)


def test_initial_plan_valid_and_schedulable():
    pl, t = planner(), topo()
    plan = pl.initial_plan(t)
    counts = plan.meta["layer_counts"]
    assert len(plan.world) == 32 and sum(counts) == 40 and counts[-1] <= counts[0]
    _, sim = pl.schedule(plan, t)
    assert not sim.deadlock and plan.meta["predicted_iteration_s"] > 0


def test_single_gpu_loss_beats_every_ablation():
    pl, t = planner(), topo()
    plan = pl.initial_plan(t)
    victim = plan.group(0, 1).devices[1]
    t2 = t.without({victim})
    new = pl.replan(plan, t2)
    g = new.group(0, 1)
    assert g is None or (g.tp == 2 and victim not in g.devices)
    assert new.meta["layer_counts"][1] < max(new.meta["layer_counts"])
    assert any(new.assignment[1][m] == 1 and plan.assignment[1][m] == 0 for m in range(16))
    pl.schedule(new, t2)
    ours = new.meta["predicted_iteration_s"]
    for kw in ({"enable_tp_shrink": False}, {"enable_repartition": False}, {"enable_migration": False}):
        assert ours <= planner(**kw).replan(plan, t2).meta["predicted_iteration_s"] + 1e-12, kw
    assert ours < planner(enable_repartition=False).replan(plan, t2).meta["predicted_iteration_s"] * 0.95


def test_tp_shrink_keeps_training_where_exclusion_stops():
    pl, t = planner(), topo()
    plan = pl.initial_plan(t)
    victims = {plan.group(0, 1).devices[1], plan.group(1, 1).devices[2]}
    t2 = t.without(victims)
    new = pl.replan(plan, t2)
    assert all(new.group(r, 1) is not None and new.group(r, 1).tp == 2 for r in range(2))
    with pytest.raises(PlanInfeasible):
        planner(enable_tp_shrink=False).replan(plan, t2)


def test_node_loss_evicts_stage_work_to_survivors():
    pl, t = planner(), topo()
    plan = pl.initial_plan(t)
    lost = {d.id for d in t.devices if d.node == "n1"}
    new = pl.replan(plan, t.without(lost))
    new.validate()
    assert not set(new.world) & lost
    missing = [(r, s) for r in range(2) for s in range(4) if new.group(r, s) is None]
    assert missing
    for r, s in missing:
        assert r not in new.assignment[s]


def test_whole_group_rebuilt_on_a_spare_node():
    pl = planner()
    t = ClusterTopology.uniform(5, 8, nodes_per_rack=1)
    plan = pl.initial_plan(t)
    spare = {d.id for d in t.devices if d.id not in plan.world}
    assert len(spare) == 8
    new = pl.replan(plan, t.without(set(plan.group(1, 2).devices)))
    g = new.group(1, 2)
    assert g is not None and g.tp == 4 and set(g.devices) <= spare


def test_fail_slow_device_goes_to_standby():
    pl, t = planner(), topo()
    plan = pl.initial_plan(t)
    slow = plan.group(1, 2).devices[0]
    new = pl.replan(plan, t.with_speeds({slow: 0.3}))
    g = new.group(1, 2)
    assert (g is None or slow not in g.devices) and slow in new.standby
    tiny = ClusterTopology.uniform(1, 4)
    pl1 = HeteroPlanner(replace(pl.cfg, num_replicas=1, num_stages=1))
    p1 = pl1.initial_plan(tiny)
    with pytest.raises(PlanInfeasible):
        pl1.replan(p1, tiny.without(set(p1.world)))


def test_plan_cache_hits_single_node_failures():
    pl, t = planner(migration_rounds=24), topo()
    plan = pl.initial_plan(t)
    cache = PlanCache(lambda p, tt: pl.replan(p, tt))
    cache.warm(plan, t, blocking=True)
    lost = {d.id for d in t.devices if d.node == "n2"}
    t0 = time.perf_counter()
    hit = cache.lookup(plan.generation, set(t.ids()) - lost, lost)
    lookup_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    fresh = pl.replan(plan, t.without(lost))
    assert hit is not None and hit.to_json() == fresh.to_json()
    assert lookup_s < (time.perf_counter() - t0) / 10
    assert cache.lookup(plan.generation, set(t.ids()) - {"n0g0"}, {"n0g0"}) is None
    assert cache.lookup(plan.generation + 1, set(t.ids()) - lost, lost) is None
    assert cache.hits == 1 and cache.misses == 2


def test_reconfiguration_cost_counts_moved_state():
    pl, t = planner(migration_rounds=24), topo()
    plan = pl.initial_plan(t)
    specs = gpt_layer_specs(LLAMA13B)
    nodes = {d.id: d.node for d in t.devices}
    same = estimate_reconfig_cost(plan, plan, specs, node_of=nodes, rebuild_s=1.0)
    assert same.bytes_moved == 0 and same.seconds == 1.0
    new = pl.replan(plan, t.without({plan.group(0, 1).devices[1]}))
    est = estimate_reconfig_cost(plan, new, specs, node_of=nodes, rebuild_s=1.0)
    assert est.bytes_moved > 0 and est.seconds > 1.0 and est.max_device_bytes <= est.bytes_moved


def test_rejoin_heals_and_grow_adds_a_replica():
    pl = planner(migration_rounds=24)
    t = ClusterTopology.uniform(4, 8, nodes_per_rack=1)
    plan = pl.initial_plan(t)
    lost = {d.id for d in t.devices if d.node == "n1"}
    degraded = pl.replan(plan, t.without(lost))
    missing = [(r, s) for r in range(2) for s in range(4) if degraded.group(r, s) is None]
    assert missing
    bigger = ClusterTopology.uniform(5, 8, nodes_per_rack=1)
    healed = pl.replan(degraded, bigger.without(lost))
    assert all(healed.group(r, s) is not None for r in range(2) for s in range(4))
    assert healed.meta["predicted_iteration_s"] < degraded.meta["predicted_iteration_s"]
    grow = planner(migration_rounds=24, max_replicas=3)
    big = ClusterTopology.uniform(6, 8, nodes_per_rack=1)
    p2 = grow.initial_plan(big)
    grown = grow.replan(p2, big)
    assert grown.num_replicas == 3 and len(grown.world) == 48
    assert grown.meta["predicted_iteration_s"] < p2.meta["predicted_iteration_s"]
