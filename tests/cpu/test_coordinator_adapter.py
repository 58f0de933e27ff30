"""Planner callback of the coordinator: PREPARE payloads, plan-cache hits, the infeasible
fallback and what-if pricing of a slow device."""

from resihp_megatron_b200.control.coordinator import ClusterView
from resihp_megatron_b200.control.membership import WorkerRecord
from resihp_megatron_b200.plan.coordinator_adapter import make_hetero_planner, make_what_if
from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan
from resihp_megatron_b200.plan.ir import schedule_from_json, validate
from resihp_megatron_b200.plan.model_spec import ModelProfile, ModelSpec
from resihp_megatron_b200.plan.planner import PlannerConfig

MODEL = ModelSpec(num_layers=8, hidden=1024, ffn=4096, num_heads=16, num_kv_heads=16, vocab=1000, seq_len=512)
PROFILE = ModelProfile(alpha=3e-6, beta=1e-10)


def cfg(**kw):
    base = dict(model=MODEL, profile=PROFILE, num_stages=2, num_replicas=2, tp=2, num_microbatches=8)
    base.update(kw)
    return PlannerConfig(**base)


def records(nodes=3, gpus=4, dead=(), slow=None):
    out = []
    for n in range(nodes):
        for g in range(gpus):
            w = f"n{n}g{g}"
            if w in dead:
                continue
            rec = WorkerRecord(w, f"n{n}", g)
            if slow and w in slow:
                rec.health["p"] = slow[w]
            out.append(rec)
    return out


def test_initial_plan_then_failure_replan():
    fn = make_hetero_planner(cfg())
    world, payload = fn(ClusterView(1, records(), [], [], None, {}, "start"))
    plan = HeteroParallelPlan.from_json(payload["plan"])
    assert plan.generation == 1 and len(world) == 8 and len(plan.standby) == 4
    assert payload["kind"] == "hetero" and payload["previous_plan"] is None and not payload["plan_cache_hit"]
    validate(plan, schedule_from_json(payload["schedule"]))
    assert set(payload["nodes"]) == {r.worker_id for r in records()}
    victim = plan.group(0, 1).devices[0]
    rec = {w: {"committed_iteration": 5} for w in world if w != victim}
    world2, payload2 = fn(ClusterView(2, records(dead={victim}), [victim], world, payload, rec, "failure"))
    plan2 = HeteroParallelPlan.from_json(payload2["plan"])
    assert victim not in world2 and plan2.generation == 2
    assert payload2["previous_plan"] == payload["plan"]
    assert payload2["recovery"]["target_iteration"] == 5 and payload2["recovery"]["restore"] is None
    validate(plan2, schedule_from_json(payload2["schedule"]))
    assert victim not in plan2.group(0, 1).devices
    assert payload2["predicted_iteration_s"] > 0 and payload2["planning_s"] >= 0


def test_whole_node_loss_hits_the_plan_cache():
    fn = make_hetero_planner(cfg())
    world, payload = fn(ClusterView(1, records(), [], [], None, {}, "start"))
    fn.cache.wait()
    plan = HeteroParallelPlan.from_json(payload["plan"])
    node = sorted({d.split("g")[0] for d in plan.world})[0]
    dead = {f"{node}g{g}" for g in range(4)}
    rec = {w: {"committed_iteration": 3} for w in world if w not in dead}
    world2, payload2 = fn(ClusterView(2, records(dead=dead), sorted(dead & set(world)), world, payload, rec, "failure"))
    assert payload2["plan_cache_hit"] and fn.cache.hits == 1
    assert not dead & set(world2)
    assert HeteroParallelPlan.from_json(payload2["plan"]).generation == 2


def test_slow_survivors_bypass_the_cache():
    fn = make_hetero_planner(cfg())
    world, payload = fn(ClusterView(1, records(), [], [], None, {}, "start"))
    fn.cache.wait()
    dead = {f"n0g{g}" for g in range(4)}
    slow = {w: 0.5 for w in world if w not in dead}
    _, payload2 = fn(ClusterView(2, records(dead=dead, slow=slow), sorted(dead & set(world)), world, payload, {},
                                 "failure"))
    assert not payload2["plan_cache_hit"]


def test_infeasible_replan_rebuilds_with_fewer_replicas():
    fn = make_hetero_planner(cfg(num_replicas=2, num_stages=2, tp=1), use_cache=False)
    world, payload = fn(ClusterView(1, records(nodes=1, gpus=4), [], [], None, {}, "start"))
    plan = HeteroParallelPlan.from_json(payload["plan"])
    dead = {plan.group(0, 1).devices[0], plan.group(1, 1).devices[0]}  # every copy of stage 1
    world2, payload2 = fn(ClusterView(2, records(nodes=1, gpus=4, dead=dead), sorted(dead), world, payload, {},
                                      "failure"))
    plan2 = HeteroParallelPlan.from_json(payload2["plan"])
    assert payload2["recovery"]["restore"] == "snapshot_or_checkpoint"
    assert not dead & set(world2) and {g.stage for g in plan2.stage_groups} == {0, 1}
    assert len(plan2.stage_groups) == 2 and plan2.generation == 2


def test_what_if_prices_a_slow_device():
    fn = make_hetero_planner(cfg(), use_cache=False)
    _, payload = fn(ClusterView(1, records(), [], [], None, {}, "start"))
    plan = HeteroParallelPlan.from_json(payload["plan"])
    slow_dev = plan.group(0, 0).devices[0]
    w = make_what_if(cfg())(payload, {slow_dev: 0.25})
    assert w.current_s > w.mitigated_s > 0
    assert w.reconfig_s > 0 and w.bytes_moved >= 0
