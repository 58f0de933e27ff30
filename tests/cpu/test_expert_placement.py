"""Expert placement: replica counts, speed-aware packing, sticky re-placement, holder groups."""

import pytest

from resihp_megatron_b200.plan.expert_placement import (ExpertPlacement, expert_dp_groups, group_time,
                                                        moved_experts, place_group, plan_expert_placement,
                                                        replica_counts, smooth_weighted_round_robin)
from resihp_megatron_b200.plan.planner import PlanInfeasible


def test_replica_counts_go_to_the_highest_load_per_copy():
    assert replica_counts([1, 1, 1], 3) == [1, 1, 1]
    assert replica_counts([8, 1, 1, 2], 6) == [3, 1, 1, 1]
    assert replica_counts([8, 1, 1, 6], 7) == [2, 1, 1, 3] or replica_counts([8, 1, 1, 6], 7) == [3, 1, 1, 2]
    assert replica_counts([9, 1], 5, max_copies=2) == [2, 2]
    with pytest.raises(PlanInfeasible):
        replica_counts([1, 1, 1], 2)


def test_hot_expert_is_replicated_and_slow_device_unloaded():
    loads = [10.0, 1, 1, 1, 1, 1]
    speeds = {"a": 1.0, "b": 1.0, "c": 0.4}
    slots = place_group(["a", "b", "c"], speeds, loads, 3)
    assert {e for v in slots.values() for e in v} == set(range(6))
    assert all(len(set(v)) == len(v) <= 3 for v in slots.values())
    assert sum(1 for v in slots.values() if 0 in v) >= 2
    singles = place_group(["a", "b", "c"], speeds, loads, 2)
    assert group_time(slots, loads, speeds) < group_time(singles, loads, speeds)

    def work(d):
        cap = {}
        for dd, es in slots.items():
            for e in es:
                cap[e] = cap.get(e, 0) + speeds[dd]
        return sum(loads[e] * speeds[d] / cap[e] for e in slots[d])

    assert work("c") < min(work("a"), work("b"))


def test_replan_after_failure_is_sticky():
    p1 = plan_expert_placement([["a", "b"], ["c", "d"]], 6)
    assert {len(p1.holders(e)) for e in range(6)} == {2}
    assert all(len(p1.group_holders(g, e)) == 1 for g in range(2) for e in range(6))
    p2 = plan_expert_placement([["a", "b", "c"]], 6, prev=p1, slots_per_device=2)
    p2.validate()
    # incumbents keep what they held; only the lost device's experts move
    assert set(p2.slots["a"]) <= set(p1.slots["a"]) and set(p2.slots["b"]) <= set(p1.slots["b"])
    assert moved_experts(p1, p2) == 1
    cold = plan_expert_placement([["c", "b", "a"]], 6, slots_per_device=2)
    assert moved_experts(p1, cold) > moved_experts(p1, p2)
    assert ExpertPlacement.from_json(p2.to_json()) == p2


def test_expert_dp_groups_and_weighted_token_split():
    p = plan_expert_placement([["a", "b"], ["c", "d"]], 4)
    groups = expert_dp_groups(p)
    assert sorted(e for es in groups.values() for e in es) == [0, 1, 2, 3]
    assert all(len(h) == 2 and len({p.group_of(d) for d in h}) == 2 for h in groups)
    split = smooth_weighted_round_robin(["x", "y"], {"y": 0.5}, 30)
    assert split.count("x") == 20 and split.count("y") == 10
    assert split == smooth_weighted_round_robin(["x", "y"], {"y": 0.5}, 30)
    assert max(len(s) for s in "".join(split).split("y")) <= 2, "smooth: no long bursts"


def test_infeasible_slot_budget_raises():
    with pytest.raises(PlanInfeasible):
        plan_expert_placement([["a"]], 4, max_slots=3)
