"""Planning core checked against independent oracles: random plans round-trip through JSON,
holder sets equal a per-element brute force, 1F1B meets its closed form, the IR validator
agrees with a naive blocking interpreter on random compute orders, zero-bubble and interleaved
schedules validate, migration never makes a plan slower, placement keeps stages off single
points of failure."""

import itertools
import random
from dataclasses import replace

import pytest

from resihp_megatron_b200.plan.cost_model import CostModel, Workload
from resihp_megatron_b200.plan.dp_migration import initial_assignment, progress_aware_migration, simulate
from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup, interleave
from resihp_megatron_b200.plan.ir import (Op, ScheduleError, compute_order_to_ir, schedule_from_json,
                                          schedule_to_json, stream_simulation, validate)
from resihp_megatron_b200.plan.model_spec import ModelProfile, ModelSpec
from resihp_megatron_b200.plan.placement import place_groups, stage_loss_exposure
from resihp_megatron_b200.plan.simulator import list_schedule, schedule_with_fallback
from resihp_megatron_b200.plan.topology import ClusterTopology
from resihp_megatron_b200.utils.intervals import even_split


def build_plan(degrees, layers=8, microbatches=8, rows=None, sp=False):
    """``degrees[r][s]``: TP degree of replica r at stage s; devices d0, d1, ... in rank order."""
    replicas, stages = len(degrees), len(degrees[0])
    per_stage = layers // stages
    groups, world = [], []
    for s in range(stages):
        for r in range(replicas):
            devs = tuple(f"d{len(world) + j}" for j in range(degrees[r][s]))
            world += devs
            groups.append(StageGroup(r, s, devs, (s * per_stage, (s + 1) * per_stage)))
    table = rows or tuple(tuple(m * replicas // microbatches for m in range(microbatches)) for _ in range(stages))
    return HeteroParallelPlan(1, tuple(world), layers, stages, replicas, tuple(groups), microbatches, table,
                              sequence_parallel=sp)


def unit_cost(f=1.0, b=2.0, w=0.5):
    return lambda key, op, mb: {"F": f, "B": b, "W": w}[op]


def free_comm(src, dst, kind):
    return 0.0


@pytest.mark.parametrize("seed", range(10))
def test_random_plans_round_trip_and_reject_corruption(seed):
    rng = random.Random(seed)
    degrees = [[rng.randint(1, 3) for _ in range(rng.randint(1, 3))] for _ in range(rng.randint(1, 3))]
    width = len(degrees[0])
    degrees = [row[:width] + [1] * (width - len(row)) for row in degrees]
    plan = build_plan(degrees, layers=2 * width, microbatches=rng.choice([2, 4, 6]), sp=rng.random() < 0.5)
    plan.validate()
    assert HeteroParallelPlan.from_json(plan.to_json()) == plan
    broken = [replace(plan, world=plan.world + ("stray",)),
              replace(plan, assignment=tuple((9,) * plan.num_microbatches for _ in range(plan.num_stages))),
              replace(plan, stage_groups=tuple(replace(g, layers=(0, 1)) for g in plan.stage_groups))]
    if width > 1 or len(degrees) > 1:
        for bad in broken:
            with pytest.raises(ValueError):
                bad.validate()


def _holder_sets_by_element(plan, stage, n):
    """Per element of a length-n dimension: the ranks holding it, one per TP partition."""
    partitions = plan.tp_slices(stage)
    sets = []
    for x in range(n):
        holders = []
        for devices in partitions:
            spans = even_split(n, len(devices))
            holders.append(plan.rank(next(d for d, (lo, hi) in zip(devices, spans) if lo <= x < hi)))
        key = tuple(sorted(holders))
        if key not in sets:
            sets.append(key)
    return sets


@pytest.mark.parametrize("tps", [((2,), (2,)), ((4,), (2,)), ((4,), (3,)), ((3,), (2,), (1,)), ((5,), (4,))])
def test_holder_sets_equal_the_per_element_brute_force(tps):
    plan = build_plan(tps, layers=1, microbatches=2)
    for n in (24, 7, 60):
        assert sorted(plan.dpshard_holder_sets(0, (n,))) == sorted(_holder_sets_by_element(plan, 0, n))


@pytest.mark.parametrize("stages,microbatches", [(2, 4), (4, 8), (3, 3)])
def test_1f1b_meets_its_closed_form(stages, microbatches):
    plan = build_plan([[1] * stages], layers=stages, microbatches=microbatches)
    res = list_schedule(plan, unit_cost(), free_comm)
    assert not res.deadlock
    assert res.makespan == pytest.approx((microbatches + stages - 1) * 3.0)  # (M + S - 1) (t_F + t_B)
    assert max(res.peak_inflight.values()) <= stages
    ir = compute_order_to_ir(plan, res.order)
    validate(plan, ir)
    assert schedule_from_json(schedule_to_json(ir)) == ir
    replay = stream_simulation(ir, duration=lambda k, ins: {Op.F: 1.0, Op.B: 2.0}.get(ins.op, 0.0))
    assert replay.complete and replay.makespan == pytest.approx(res.makespan)


def _naive_runs_to_completion(ir, plan) -> bool:
    """Blocking interpreter: sends post into per-channel FIFOs; a receive must find its message
    at the head of its channel."""
    queues = {}
    position = {k: 0 for k in ir}
    progressed = True
    while progressed:
        progressed = False
        for key, stream in ir.items():
            while position[key] < len(stream):
                ins = stream[position[key]]
                if ins.op in (Op.SEND_ACT, Op.SEND_GRAD):
                    queues.setdefault((key, plan.physical_key(*ins.peer), ins.op.value[1]), []).append(ins.mb)
                elif ins.op in (Op.RECV_ACT, Op.RECV_GRAD):
                    q = queues.get((plan.physical_key(*ins.peer), key, ins.op.value[1]), [])
                    if not q or q[0] != ins.mb:
                        break
                    q.pop(0)
                position[key] += 1
                progressed = True
    return all(position[k] == len(s) for k, s in ir.items())


def _random_orders(plan, rng):
    """Per slot: a random interleaving of its F and B ops, each B after its own F."""
    orders = {}
    for g in plan.stage_groups:
        mbs = plan.microbatches_of(g.replica, g.stage)
        pending_f, pending_b, order = list(mbs), [], []
        while pending_f or pending_b:
            if pending_b and (not pending_f or rng.random() < 0.5):
                order.append(("B", pending_b.pop(rng.randrange(len(pending_b)))))
            else:
                mb = pending_f.pop(0 if rng.random() < 0.7 else rng.randrange(len(pending_f)))
                order.append(("F", mb))
                pending_b.append(mb)
        orders[(g.replica, g.stage)] = order
    return orders


@pytest.mark.parametrize("seed", range(40))
def test_ir_validator_agrees_with_a_naive_interpreter(seed):
    rng = random.Random(seed)
    plan = build_plan([[1] * rng.choice([2, 3])], layers=6, microbatches=rng.choice([2, 3]))
    ir = compute_order_to_ir(plan, _random_orders(plan, rng))
    try:
        validate(plan, ir)
        accepted = True
    except ScheduleError:
        accepted = False
    assert accepted == _naive_runs_to_completion(ir, plan)


def test_zero_bubble_places_one_w_after_every_b():
    plan = build_plan([[1, 1, 1]], layers=6, microbatches=6)
    res = list_schedule(plan, unit_cost(1.0, 1.0), free_comm, split_backward=True)
    ir = compute_order_to_ir(plan, res.order)
    validate(plan, ir, split_backward=True)
    for stream in ir.values():
        ops = [(i.op, i.mb) for i in stream if i.op in (Op.B, Op.W)]
        for mb in range(6):
            assert ops.index((Op.B, mb)) < ops.index((Op.W, mb))


def test_interleaved_plan_schedules_and_folds_back():
    plan = interleave(build_plan([[1, 1]], layers=8, microbatches=4), 2)
    plan.validate()
    assert (plan.num_stages, plan.vpp) == (4, 2)
    res = schedule_with_fallback(plan, unit_cost(), free_comm)
    assert not res.deadlock
    validate(plan, compute_order_to_ir(plan, res.order))
    folded = plan.physical()
    assert folded.num_stages == 2 and sum(g.num_layers for g in folded.groups_at(0)[:1]) == 4


def _costs(plan, speeds):
    spec = ModelSpec(num_layers=plan.num_layers, hidden=1024, ffn=4096, num_heads=16, num_kv_heads=16, vocab=1000,
                     seq_len=1024)
    return CostModel(plan, spec, ModelProfile(alpha=1e-6, beta=0.0, last_stage_extra_layers=0.0),
                     Workload.uniform(plan.num_microbatches, 1024), speeds, {d: d for d in plan.world})


@pytest.mark.parametrize("slow", [0.3, 0.5, 0.8])
def test_migration_never_slows_a_plan_and_relieves_the_slow_group(slow):
    plan = build_plan([[1, 1, 1]] * 3, layers=6, microbatches=12)
    speeds = dict.fromkeys(plan.world, 1.0)
    speeds[plan.group(1, 1).devices[0]] = slow
    res = progress_aware_migration(plan, _costs(plan, speeds), max_rounds=32)
    assert res.makespan <= res.initial_makespan + 1e-12
    final = replace(plan, assignment=res.assignment)
    final.validate()
    validate(final, compute_order_to_ir(final, res.sim.order))
    assert res.assignment[1].count(1) <= plan.assignment[1].count(1)  # the slow group never gains work


def test_eviction_respects_memory_caps():
    full = build_plan([[1, 1, 1]] * 3, layers=6, microbatches=12)
    groups = tuple(g for g in full.stage_groups if (g.replica, g.stage) != (1, 2))
    world = tuple(d for d in full.world if any(d in g.devices for g in groups))
    table = initial_assignment(list(groups), 3, 12, lambda key: 1.0)
    assert 1 not in table[2] and sorted(table[2]) == sorted(table[2])
    plan = replace(full, stage_groups=groups, world=world, assignment=table)
    plan.validate()
    costs = _costs(plan, dict.fromkeys(world, 1.0))
    caps = {(g.replica, g.stage): 4 for g in groups}
    res = progress_aware_migration(plan, costs, mem_cap=caps)
    sim = simulate(replace(plan, assignment=res.assignment), costs)
    assert all(sim.peak_inflight[k] <= caps[k] for k in caps)


def test_spread_placement_survives_every_single_node_loss():
    topo = ClusterTopology.uniform(4, 8, nodes_per_rack=2)
    spread = place_groups(topo, num_replicas=2, num_stages=4, tp=4, strategy="spread")
    packed = place_groups(topo, num_replicas=2, num_stages=4, tp=4, strategy="megatron")
    assert stage_loss_exposure(spread, topo) == 0.0 < stage_loss_exposure(packed, topo)
    devices = [d for v in spread.values() for d in v]
    assert len(devices) == len(set(devices)) == 32
    node_of = {d.id: d.node for d in topo.devices}
    for key, devs in spread.items():  # every TP group is inside one node (NVLink domain)
        assert len({node_of[d] for d in devs}) == 1
    for node in {d.node for d in topo.devices}:  # brute force of the exposure measure
        for stage in range(4):
            holders = [devs for (r, s), devs in spread.items() if s == stage]
            assert not all(any(node_of[d] == node for d in devs) for devs in holders)
