"""Cluster simulator checked against closed forms and brute force: trace statistics,
the integer micro-batch capacity, policy throughput after a loss, and the time accounting."""

import itertools
import math
import random

import pytest

from resihp_megatron_b200.sim.cluster import (ClusterState, JobConfig, baseline_params, ideal_params,
                                              integer_capacity, resihp_params, simulate)
from resihp_megatron_b200.sim.traces import LLAMA3_UNEXPECTED, Event, TraceConfig, expected_failures, generate


def test_trace_rates_sizes_and_determinism():
    total = sum(n for n, _ in LLAMA3_UNEXPECTED.values())
    assert total == 419
    assert expected_failures(16384, 54) == pytest.approx(total)
    assert expected_failures(1024, 10) == pytest.approx(total * (1024 / 16384) * (10 / 54))
    cfg = TraceConfig(gpus=16384, slow_per_gpu_day=0.0, seed=7)
    events = generate(cfg)
    assert abs(len(events) - total) < 4 * math.sqrt(total)  # Poisson: within 4 sigma
    sizes = {"gpu": 1, "node": cfg.gpus_per_node, "network": 2 * cfg.gpus_per_node, "job": 0}
    assert all(len(e.targets) == sizes[e.domain] and all(0 <= g < cfg.gpus for g in e.targets) for e in events)
    assert [e.t for e in events] == sorted(e.t for e in events)
    assert generate(cfg) == events and generate(TraceConfig(gpus=16384, slow_per_gpu_day=0.0, seed=8)) != events


def _capacity_by_search(caps, m):
    """The least T with sum floor(T c) >= m over all completion instants k / c."""
    instants = sorted({k / c for c in caps if c > 0 for k in range(1, m + 1)})
    t = next(t for t in instants if sum(math.floor(t * c + 1e-9) for c in caps) >= m)
    return m / t


@pytest.mark.parametrize("seed", range(15))
def test_integer_capacity_matches_exhaustive_search(seed):
    rng = random.Random(seed)
    caps = [rng.choice([0.0, 0.25, 0.5, 0.75, 0.9, 1.0]) for _ in range(rng.randint(1, 5))]
    m = rng.randint(1, 30)
    if not any(caps):
        assert integer_capacity(caps, m) == 0.0
    else:
        assert integer_capacity(caps, m) == pytest.approx(_capacity_by_search(caps, m))


def test_integer_capacity_closed_forms():
    assert integer_capacity([1.0] * 4, 16) == 4  # even split: no loss
    assert integer_capacity([1.0] * 3, 16) == pytest.approx(16 / 6)  # ceil(16/3) = 6 rounds
    assert integer_capacity([1.0, 1.0, 0.5], 10) == pytest.approx(2.5)


def test_after_one_gpu_loss_resihp_keeps_more_than_dropping_a_replica():
    job = JobConfig(gpus=1024, tp=8, pp=16)
    kept = {}
    for policy in [resihp_params(job), *baseline_params(job)]:
        st = ClusterState(job, policy)
        st.fail([5], math.inf)
        st.refresh([5])
        kept[policy.name] = st.throughput()
    dp = job.dp
    assert kept["torchft"] == pytest.approx((dp - 1) / dp)  # one replica gone, batch shrinks
    assert kept["ResiHP"] > kept["torchft-bp"]
    assert kept["ResiHP"] >= kept["ReCycle"] - 1e-9


def test_spare_node_covers_a_failed_node():
    job = JobConfig(gpus=1024, tp=8, pp=16, spare_nodes=1)
    st = ClusterState(job, baseline_params(job)[1])
    degrading, taken = st.fail(list(range(8)), 100.0)
    assert taken == 1 and degrading == [] and not st.lost
    assert st.repair(list(range(8)), 100.0) == list(range(8)) and st.spares_free == 1


def test_accounting_of_one_failure():
    job = JobConfig(gpus=1024, tp=8, pp=16, iteration_s=10.0)
    day = 86400.0
    for policy in [ideal_params(), resihp_params(job), *baseline_params(job)]:
        assert simulate([], job, policy, day).ettr == pytest.approx(1.0)
    failure = [Event(4000.0, "fail", "gpu", "faulty_gpu", (17,), 7200.0)]
    res = {p.name: simulate(failure, job, p, day) for p in [resihp_params(job), *baseline_params(job)]}
    assert res["ResiHP"].ettr > res["torchft-bp"].ettr > res["NVRx"].ettr
    assert res["ResiHP"].lost_s <= job.iteration_s < res["NVRx"].lost_s  # online vs restart from checkpoint
    for r in res.values():  # every second of the horizon is progress, rolled back, degraded or down
        assert r.progress_s + r.lost_s + r.degraded_loss_s + r.downtime_s == pytest.approx(day, rel=1e-9)
    slow = [Event(100.0, "slow", "gpu", "fail_slow", (3,), 5000.0, 2.0)]
    r = simulate(slow, job, resihp_params(job), day)
    assert 0.97 < r.ettr < 1.0 and r.events == 1  # detected after three iterations, then migrated
