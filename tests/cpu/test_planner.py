"""The joint planner checked by properties over many failure scenarios and by brute force:
every replanned plan is valid and avoids the failed devices; the full planner is never slower
than any of its ablations; a weakened TP group gets the Eq. 4 optimum over its survivors; the
plan cache returns exactly the plan a fresh replan computes; the reconfiguration price counts
exactly the elements a device does not already hold."""

import itertools
import random
import time
from dataclasses import replace

import pytest

from resihp_megatron_b200.plan.model_spec import ModelProfile, ModelSpec
from resihp_megatron_b200.plan.plan_cache import PlanCache
from resihp_megatron_b200.plan.planner import HeteroPlanner, PlanInfeasible, PlannerConfig
from resihp_megatron_b200.plan.reconfig_cost import estimate_reconfig_cost, gpt_layer_specs, layer_of_key
from resihp_megatron_b200.plan.topology import ClusterTopology
from resihp_megatron_b200.state.layer_registry import holdings
from resihp_megatron_b200.utils.intervals import intersect

MODEL = ModelSpec(num_layers=40, hidden=5120, ffn=13824, num_heads=40, num_kv_heads=40, vocab=32000, seq_len=4096)
PROFILE = ModelProfile(alpha=3.0e-6, beta=1.0e-10, last_stage_extra_layers=1.0)
ABLATIONS = ({"enable_tp_shrink": False}, {"enable_repartition": False}, {"enable_migration": False})


def make_planner(**overrides) -> HeteroPlanner:
    cfg = PlannerConfig(model=MODEL, profile=PROFILE, num_stages=4, num_replicas=2, tp=4, num_microbatches=16,
                        mem_capacity=80e9, migration_rounds=24)
    return HeteroPlanner(replace(cfg, **overrides))


@pytest.fixture(scope="module")
def baseline():
    planner, topo = make_planner(), ClusterTopology.uniform(4, 8, nodes_per_rack=2)
    return planner, topo, planner.initial_plan(topo)


def test_initial_plan(baseline):
    planner, topo, plan = baseline
    counts = plan.meta["layer_counts"]
    assert sum(counts) == MODEL.num_layers and len(plan.world) == 32
    assert counts[-1] <= counts[0]  # the last stage also carries the LM head
    _, sim = planner.schedule(plan, topo)
    assert not sim.deadlock and plan.meta["predicted_iteration_s"] > 0


@pytest.mark.parametrize("seed", range(6))
def test_random_failures_replan_to_valid_plans_no_slower_than_ablations(baseline, seed):
    planner, topo, plan = baseline
    rng = random.Random(seed)
    used = list(plan.world)
    victims = set(rng.sample(used, rng.choice([1, 1, 2])))
    degraded = topo.without(victims)
    try:
        new = planner.replan(plan, degraded)
    except PlanInfeasible:
        pytest.skip("this loss leaves a stage without any feasible group")
    new.validate()
    assert not victims & set(new.world)
    assert all(new.groups_at(s) for s in range(new.num_stages))
    planner.schedule(new, degraded)
    ours = new.meta["predicted_iteration_s"]
    assert ours >= plan.meta["predicted_iteration_s"] - 1e-12  # losing hardware never helps
    for kw in ABLATIONS:
        try:
            theirs = make_planner(**kw).replan(plan, degraded).meta["predicted_iteration_s"]
        except PlanInfeasible:
            continue
        assert ours <= theirs + 1e-12, kw


def _eq4_best(profile, survivors: int, degrees) -> int:
    """Brute force of Eq. 4 for equal-speed survivors: the degree maximising k * eff(k)."""
    scores = {k: profile.group_speed(k, 1.0) for k in degrees if k <= survivors}
    top = max(scores.values())
    return max(k for k, s in scores.items() if s >= top - 1e-12)


def test_weakened_group_gets_the_eq4_optimum(baseline):
    planner, topo, plan = baseline
    victim = plan.group(0, 1).devices[1]
    new = planner.replan(plan, topo.without({victim}))
    group = new.group(0, 1)
    if group is not None:  # kept (not evicted): its degree is the brute-force optimum
        degrees = [k for k in range(1, 5) if MODEL.tp_feasible(k) and k >= planner.mem.min_tp(
            plan.meta["layer_counts"][1], 1)]
        assert group.tp == _eq4_best(PROFILE, 3, degrees) and victim not in group.devices


def test_shrink_keeps_a_stage_alive_where_exclusion_cannot(baseline):
    planner, topo, plan = baseline
    victims = {plan.group(0, 1).devices[1], plan.group(1, 1).devices[2]}
    new = planner.replan(plan, topo.without(victims))
    assert all(new.group(r, 1) is not None and new.group(r, 1).tp < 4 for r in range(2))
    with pytest.raises(PlanInfeasible):
        make_planner(enable_tp_shrink=False).replan(plan, topo.without(victims))


def test_a_lost_group_is_rebuilt_on_spare_hardware():
    planner = make_planner()
    topo = ClusterTopology.uniform(5, 8, nodes_per_rack=1)
    plan = planner.initial_plan(topo)
    spare = set(topo.ids()) - set(plan.world)
    rebuilt = planner.replan(plan, topo.without(set(plan.group(1, 2).devices))).group(1, 2)
    assert rebuilt is not None and rebuilt.tp == 4 and set(rebuilt.devices) <= spare


def test_plan_cache_returns_the_fresh_replan(baseline):
    planner, topo, plan = baseline
    cache = PlanCache(lambda p, t: planner.replan(p, t))
    cache.warm(plan, topo, blocking=True)
    for node in sorted({d.node for d in topo.devices}):
        lost = {d.id for d in topo.devices if d.node == node}
        started = time.perf_counter()
        hit = cache.lookup(plan.generation, set(topo.ids()) - lost, lost)
        lookup_s = time.perf_counter() - started
        try:
            fresh = planner.replan(plan, topo.without(lost))
        except PlanInfeasible:
            assert hit is None
            continue
        assert hit is not None and hit.to_json() == fresh.to_json() and lookup_s < 0.01
    assert cache.lookup(plan.generation + 1, set(topo.ids()) - lost, lost) is None  # stale generation


def _elements(spec, span) -> int:
    n = 1
    for d in spec.local_shape(span):
        n *= d
    return n


def test_reconfiguration_price_counts_exactly_the_missing_elements(baseline):
    planner, topo, plan = baseline
    specs = gpt_layer_specs(MODEL)
    nodes = {d.id: d.node for d in topo.devices}
    assert estimate_reconfig_cost(plan, plan, specs, node_of=nodes, rebuild_s=1.0).bytes_moved == 0
    new = planner.replan(plan, topo.without({plan.group(0, 1).devices[1]}))
    est = estimate_reconfig_cost(plan, new, specs, node_of=nodes, rebuild_s=1.0, bytes_per_elem=14)
    before, after = holdings(plan, specs, layer_of_key), holdings(new, specs, layer_of_key)
    survivors = set(plan.world) & set(new.world)
    missing = 0
    for key, pairs in after.items():
        for dev, want in pairs:
            had = [span for d, span in before.get(key, []) if d == dev and d in survivors]
            kept = sum(_elements(specs[key], o) for o in (intersect(h, want) for h in had) if o is not None)
            missing += _elements(specs[key], want) - kept
    assert est.bytes_moved == 14 * missing > 0
    assert est.seconds > 1.0 and est.max_device_bytes <= 2 * est.bytes_moved


def test_rejoin_heals_and_grow_adds_a_whole_replica():
    planner = make_planner()
    topo = ClusterTopology.uniform(4, 8, nodes_per_rack=1)
    plan = planner.initial_plan(topo)
    lost = {d.id for d in topo.devices if d.node == "n1"}
    degraded = planner.replan(plan, topo.without(lost))
    assert any(degraded.group(r, s) is None for r, s in itertools.product(range(2), range(4)))
    healed = planner.replan(degraded, ClusterTopology.uniform(5, 8, nodes_per_rack=1).without(lost))
    assert all(healed.group(r, s) is not None for r, s in itertools.product(range(2), range(4)))
    assert healed.meta["predicted_iteration_s"] < degraded.meta["predicted_iteration_s"]
    grower = make_planner(max_replicas=3)
    big = ClusterTopology.uniform(6, 8, nodes_per_rack=1)
    start = grower.initial_plan(big)
    grown = grower.replan(start, big)
    assert grown.num_replicas == 3 and len(grown.world) == 48
    assert grown.meta["predicted_iteration_s"] < start.meta["predicted_iteration_s"]
