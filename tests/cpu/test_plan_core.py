"""Planning core: plan validation / JSON, shard-aligned DP groups, 1F1B closed form, IR
validation, TP selection, min-max partition, migration, placement."""

from dataclasses import replace

import pytest

from resihp_megatron_b200.plan.cost_model import CostModel, Workload
from resihp_megatron_b200.plan.dp_migration import initial_assignment, progress_aware_migration, simulate
from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup, dpshard_group_name, interleave
from resihp_megatron_b200.plan.ir import (Instr, Op, ScheduleError, compute_order_to_ir, schedule_from_json,
                                          schedule_to_json, stream_simulation, validate)
from resihp_megatron_b200.plan.layer_partition import counts_to_ranges, partition_layers
from resihp_megatron_b200.plan.model_spec import ModelProfile, ModelSpec
from resihp_megatron_b200.plan.placement import place_groups, stage_loss_exposure
from resihp_megatron_b200.plan.simulator import list_schedule, schedule_with_fallback
from resihp_megatron_b200.plan.topology import ClusterTopology
from resihp_megatron_b200.plan.tp_select import feasible_degrees, min_tp_for_memory, select_subgroup


def make_plan(tps=((2, 2), (2, 2)), layers=8, M=8, assignment=None, sp=False):
    """``tps[r][s]`` = TP degree of replica r at stage s; devices are numbered in rank order."""
    R, S = len(tps), len(tps[0])
    groups, world, n = [], [], 0
    per = layers // S
    for s in range(S):
        for r in range(R):
            devs = tuple(f"d{n + j}" for j in range(tps[r][s]))
            n += tps[r][s]
            world += devs
            groups.append(StageGroup(r, s, devs, (s * per, (s + 1) * per)))
    if assignment is None:
        assignment = tuple(tuple(m * R // M for m in range(M)) for _ in range(S))
    return HeteroParallelPlan(1, tuple(world), layers, S, R, tuple(groups), M, assignment, sequence_parallel=sp)


def fixed_cost(f=1.0, b=2.0, w=0.5):
    return lambda key, op, mb: {"F": f, "B": b, "W": w}[op]


def no_comm(a, b, k):
    return 0.0


def test_plan_validation_and_json_roundtrip():
    p = make_plan()
    p.validate()
    assert HeteroParallelPlan.from_json(p.to_json()) == p
    with pytest.raises(ValueError):
        replace(p, assignment=((0,) * 8, (5,) * 8)).validate()
    with pytest.raises(ValueError):
        replace(p, world=p.world + ("ghost",)).validate()
    bad_layers = tuple(replace(g, layers=(0, 4)) for g in p.stage_groups)
    with pytest.raises(ValueError):
        replace(p, stage_groups=bad_layers).validate()


def test_uniform_tp_gives_plain_dp_groups():
    p = make_plan(tps=((2, 2), (2, 2)))
    assert p.dpshard_holder_sets(0, (24, 8)) == [(0, 2), (1, 3)]


def test_heterogeneous_tp_groups_follow_the_refinement():
    p = make_plan(tps=((4,), (2,)))
    assert p.dpshard_holder_sets(0, (24,)) == [(0, 4), (1, 4), (2, 5), (3, 5)]
    p3 = make_plan(tps=((4,), (3,)))
    assert p3.dpshard_holder_sets(0, (24,)) == [(0, 4), (1, 4), (1, 5), (2, 5), (2, 6), (3, 6)]
    names = {s.name for s in p3.group_specs((24,))}
    assert "tp/r0/s0" in names and dpshard_group_name(0, (1, 5)) in names


def test_1f1b_makespan_closed_form_and_ir():
    S, M = 4, 8
    p = make_plan(tps=((1,) * S,), layers=8, M=M)
    res = list_schedule(p, fixed_cost(), no_comm)
    assert not res.deadlock
    assert res.makespan == pytest.approx((M + S - 1) * 3.0)
    assert max(res.peak_inflight.values()) <= S
    ir = compute_order_to_ir(p, res.order)
    validate(p, ir)
    assert schedule_from_json(schedule_to_json(ir)) == ir
    sim = stream_simulation(ir, duration=lambda k, ins: {Op.F: 1.0, Op.B: 2.0}.get(ins.op, 0.0))
    assert sim.complete and sim.makespan == pytest.approx(res.makespan)


def test_zero_bubble_schedules_every_w():
    p = make_plan(tps=((1, 1, 1),), layers=6, M=6)
    res = list_schedule(p, fixed_cost(1.0, 1.0), no_comm, split_backward=True)
    ir = compute_order_to_ir(p, res.order)
    validate(p, ir, split_backward=True)
    assert sum(1 for i in ir[(0, 2)] if i.op == Op.W) == 6


def test_interleaved_schedule_validates():
    p = interleave(make_plan(tps=((1, 1),), layers=8, M=4), 2)
    p.validate()
    assert p.num_stages == 4 and p.vpp == 2
    res = schedule_with_fallback(p, fixed_cost(), no_comm)
    assert not res.deadlock
    validate(p, compute_order_to_ir(p, res.order))
    assert p.physical().num_stages == 2


def test_validator_catches_fifo_violation_and_deadlock():
    p = make_plan(tps=((1, 1),), layers=4, M=2)
    ir = compute_order_to_ir(p, list_schedule(p, fixed_cost(), no_comm).order)
    s0 = list(ir[(0, 0)])
    sends = [i for i, ins in enumerate(s0) if ins.op == Op.SEND_ACT]
    s0[sends[0]], s0[sends[1]] = s0[sends[1]], s0[sends[0]]
    with pytest.raises(ScheduleError):
        validate(p, {**ir, (0, 0): s0})
    dead = {(0, 0): [Instr(Op.RECV_GRAD, 0, (0, 1)), Instr(Op.SEND_ACT, 0, (0, 1))],
            (0, 1): [Instr(Op.RECV_ACT, 1, (0, 0)), Instr(Op.SEND_GRAD, 0, (0, 0))]}
    assert not stream_simulation(dead).complete


def test_tp_selection_allows_non_power_of_two():
    m = ModelSpec(num_layers=32, hidden=4096, ffn=12288, num_heads=48, num_kv_heads=12, vocab=32000, seq_len=4096)
    assert feasible_degrees(m, 8) == [1, 2, 3, 4, 6]
    assert feasible_degrees(m, 8, power_of_two_only=True) == [1, 2, 4]
    c = select_subgroup([("a", 1.0), ("b", 1.0), ("c", 1.0), ("d", 0.3)], [1, 2, 4])
    assert c.tp == 2 and c.score == pytest.approx(2.0) and set(c.standby) == {"c", "d"}
    assert select_subgroup([("a", 1.0), ("b", 1.0), ("c", 1.0), ("d", 0.9)], [1, 2, 4]).tp == 4
    assert select_subgroup([("a", 1.0), ("b", 1.0), ("c", 1.0)], feasible_degrees(m, 3)).tp == 3
    assert min_tp_for_memory(m, 32, 80e9, inflight=1) in (1, 2)
    assert min_tp_for_memory(m, 32, 1e9, inflight=1) is None


def test_layer_partition_min_max():
    assert partition_layers(12, [1.0, 0.4, 1.0]) == [5, 2, 5]
    assert partition_layers(12, [1.0, 1.0, 1.0]) == [4, 4, 4]
    assert partition_layers(12, [1.0, 1.0, 1.0], max_layers=[3, 6, 6]) == [3, 5, 4]
    counts = partition_layers(16, [1.0] * 4, last_extra=2.0)
    assert counts[-1] < counts[0]
    assert counts_to_ranges([2, 3]) == [(0, 2), (2, 5)]
    with pytest.raises(ValueError):
        partition_layers(2, [1, 1, 1])


def _cm(plan, speeds):
    model = ModelSpec(num_layers=plan.num_layers, hidden=1024, ffn=4096, num_heads=16, num_kv_heads=16, vocab=1000,
                      seq_len=1024)
    prof = ModelProfile(alpha=1e-6, beta=0.0, last_stage_extra_layers=0.0)
    return CostModel(plan, model, prof, Workload.uniform(plan.num_microbatches, 1024), speeds,
                     {d: d for d in plan.world})


def test_migration_mitigates_a_slow_group():
    p = make_plan(tps=((1, 1, 1), (1, 1, 1), (1, 1, 1)), layers=6, M=12)
    speeds = {d: 1.0 for d in p.world}
    speeds[p.group(1, 1).devices[0]] = 0.5
    res = progress_aware_migration(p, _cm(p, speeds), max_rounds=32)
    assert res.makespan < res.initial_makespan * 0.95
    moved = [m for m in range(12) if res.assignment[1][m] != p.assignment[1][m]]
    assert moved and all(p.assignment[1][m] == 1 for m in moved)
    final = replace(p, assignment=res.assignment)
    validate(final, compute_order_to_ir(final, res.sim.order))


def test_fail_stop_eviction_respects_memory_caps():
    full = make_plan(tps=((1, 1, 1), (1, 1, 1), (1, 1, 1)), layers=6, M=12)
    groups = tuple(g for g in full.stage_groups if not (g.replica == 1 and g.stage == 2))
    world = tuple(d for d in full.world if d in {x for g in groups for x in g.devices})
    assign = initial_assignment(list(groups), 3, 12, lambda k: 1.0)
    assert 1 not in assign[2] and assign[0].count(1) == 4
    p = replace(full, stage_groups=groups, world=world, assignment=assign)
    p.validate()
    cm = _cm(p, {d: 1.0 for d in world})
    caps = {(g.replica, g.stage): 4 for g in groups}
    res = progress_aware_migration(p, cm, mem_cap=caps)
    final = replace(p, assignment=res.assignment)
    sim = simulate(final, cm)
    assert all(sim.peak_inflight[k] <= caps[k] for k in caps)
    validate(final, compute_order_to_ir(final, sim.order))


def test_spread_placement_never_loses_a_whole_stage_to_one_node():
    topo = ClusterTopology.uniform(4, 8, nodes_per_rack=2)
    spread = place_groups(topo, num_replicas=2, num_stages=4, tp=4, strategy="spread")
    packed = place_groups(topo, num_replicas=2, num_stages=4, tp=4, strategy="megatron")
    assert stage_loss_exposure(spread, topo) == 0.0
    assert stage_loss_exposure(packed, topo) == 1.0
    assert len({d for v in spread.values() for d in v}) == 32
