"""Expert placement checked by properties and small brute-force oracles, not by the reference's
own expectations."""

import itertools
import random

import pytest

from resihp_megatron_b200.plan.expert_placement import (ExpertPlacement, expert_dp_groups, group_time,
                                                        moved_experts, place_group, plan_expert_placement,
                                                        replica_counts, smooth_weighted_round_robin)
from resihp_megatron_b200.plan.planner import PlanInfeasible


def _minmax_copies_oracle(loads, slots, cap):
    """Every count vector with the same total: the optimum of max(load/copies)."""
    best = None
    for counts in itertools.product(range(1, cap + 1), repeat=len(loads)):
        if sum(counts) == slots:
            v = max(l / c for l, c in zip(loads, counts))
            best = v if best is None else min(best, v)
    return best


@pytest.mark.parametrize("seed", range(12))
def test_replica_counts_minimise_the_worst_load_per_copy(seed):
    rng = random.Random(seed)
    loads = [rng.choice([1.0, 2.0, 3.0, 5.0, 8.0]) for _ in range(rng.randint(2, 4))]
    slots = rng.randint(len(loads), 3 * len(loads))
    cap = rng.choice([None, 3])
    counts = replica_counts(loads, slots, max_copies=cap)
    limit = cap or slots
    assert all(1 <= c <= limit for c in counts)
    if sum(counts) == slots:  # not clipped by the copy cap
        got = max(l / c for l, c in zip(loads, counts))
        assert got == pytest.approx(_minmax_copies_oracle(loads, slots, limit))
    with pytest.raises(PlanInfeasible):
        replica_counts(loads, len(loads) - 1)


def test_group_time_is_the_speed_proportional_bottleneck():
    # expert 0 split over a (speed 1) and b (speed 3): each holder spends 8 / 4 = 2; b adds expert 1: 3 / 3
    assert group_time({"a": (0,), "b": (0, 1)}, [8.0, 3.0], {"a": 1.0, "b": 3.0}) == pytest.approx(3.0)


@pytest.mark.parametrize("seed", range(8))
def test_placement_invariants_and_slow_device_relief(seed):
    rng = random.Random(100 + seed)
    devices = [f"d{i}" for i in range(rng.randint(2, 4))]
    E = rng.randint(len(devices), 2 * len(devices))
    loads = [rng.choice([1.0, 1.0, 4.0]) for _ in range(E)]
    speeds = {d: 1.0 for d in devices}
    per_dev = -(-E // len(devices)) + 1
    slots = place_group(devices, speeds, loads, per_dev)
    assert set().union(*map(set, slots.values())) == set(range(E))
    assert all(len(v) == len(set(v)) <= per_dev for v in slots.values())
    slow = dict(speeds, **{devices[0]: 0.25})
    relieved = place_group(devices, slow, loads, per_dev)
    # a slowed device never gets more expert work than under uniform speeds' placement
    assert group_time(relieved, loads, slow) <= group_time(slots, loads, slow) + 1e-12


def test_replan_keeps_incumbent_copies():
    first = plan_expert_placement([["a", "b"], ["c", "d"]], 6)
    assert all(len(first.group_holders(g, e)) == 1 for g in range(2) for e in range(6))
    second = plan_expert_placement([["a", "b", "c"]], 6, prev=first, slots_per_device=2)
    second.validate()
    assert set(second.slots["a"]) <= set(first.slots["a"]) and set(second.slots["b"]) <= set(first.slots["b"])
    # only what the leaver (d) held, plus what c lacks, is new; a cold placement moves more
    cold = plan_expert_placement([["c", "b", "a"]], 6, slots_per_device=2)
    assert moved_experts(first, second) < moved_experts(first, cold)
    assert ExpertPlacement.from_json(second.to_json()) == second


def test_expert_dp_groups_cover_every_expert_once():
    p = plan_expert_placement([["a", "b"], ["c", "d"]], 4)
    groups = expert_dp_groups(p)
    assert sorted(e for es in groups.values() for e in es) == [0, 1, 2, 3]
    for holders, experts in groups.items():
        assert all(p.holders(e) == list(holders) for e in experts)
        assert len({p.group_of(d) for d in holders}) == 2  # one copy per EP group


@pytest.mark.parametrize("weights", [(1.0, 0.5), (1.0, 1.0, 0.3), (0.7, 0.2)])
def test_smooth_round_robin_is_proportional_and_smooth(weights):
    names = [f"h{i}" for i in range(len(weights))]
    speeds = dict(zip(names, weights))
    w = [max(1, round(10 * x)) for x in weights]
    period = sum(w)
    seq = smooth_weighted_round_robin(names, speeds, 3 * period)
    for name, wi in zip(names, w):
        assert seq.count(name) == 3 * wi  # exact shares over whole periods
        # smoothness: over any window of one period, a holder's count is within one of its share
        for s in range(len(seq) - period + 1):
            assert abs(seq[s:s + period].count(name) - wi) <= 1
    assert seq == smooth_weighted_round_robin(names, speeds, 3 * period)
    assert smooth_weighted_round_robin(["only"], {}, 4) == ["only"] * 4


def test_infeasible_slot_budget_raises():
    with pytest.raises(PlanInfeasible):
        plan_expert_placement([["a"]], 4, max_slots=3)


def test_receive_capacity_is_rank_independent_and_bounds_every_layout():
    """The symmetric heap's receive segments have one size on every rank, also when a
    speed-weighted placement gives ranks different expert counts, and that size bounds what any
    rank can receive: for every count table where each source routes at most T rows to each
    expert, the rows landing on a rank fit."""
    import random

    from resihp_megatron_b200.parallel.moe_ep import receive_capacity, replica_cycles, replica_layout

    rng = random.Random(0)
    for _ in range(200):
        world, E, T = rng.choice([2, 4, 8]), 8, rng.randint(1, 64)
        holders = [[rng.randrange(world)] for _ in range(E)]
        if rng.random() < 0.5:  # a replicated expert
            e = rng.randrange(E)
            holders[e] = sorted(set(holders[e] + [rng.randrange(world)]))
        cap = receive_capacity(holders, world, T)
        assert all(cap == receive_capacity(holders, world, T) for _ in range(world))
        cycles = replica_cycles(holders)
        table = [[rng.randint(0, T) for _ in range(E)] for _ in range(world)]
        for me in range(world):
            _, ranges = replica_layout(table, cycles, me, world)
            assert sum(n for _, n in ranges) <= cap
