"""Cluster simulator: trace statistics, integer micro-batch capacity, policy throughput and
accounting."""

import math

import pytest

from resihp_megatron_b200.sim.cluster import (ClusterState, JobConfig, baseline_params, ideal_params,
                                              integer_capacity, resihp_params, simulate)
from resihp_megatron_b200.sim.traces import LLAMA3_UNEXPECTED, Event, TraceConfig, expected_failures, generate


def test_trace_follows_llama3_rates():
    assert sum(c for c, _ in LLAMA3_UNEXPECTED.values()) == 419
    assert expected_failures(16384, 54) == pytest.approx(419)
    cfg = TraceConfig(gpus=16384, slow_per_gpu_day=0.0)
    events = generate(cfg)
    assert abs(len(events) - 419) < 4 * math.sqrt(419)
    for e in events:
        assert len(e.targets) == {"gpu": 1, "node": 8, "network": 16, "job": 0}[e.domain]
    assert generate(cfg) == events and all(a.t <= b.t for a, b in zip(events, events[1:]))


def test_integer_capacity_is_exact():
    assert integer_capacity([1.0] * 4, 16) == 4
    assert integer_capacity([1.0] * 3, 16) == pytest.approx(16 / 6)
    assert integer_capacity([1.0, 1.0, 0.5], 10) == pytest.approx(2.5)
    assert integer_capacity([0.0, 0.0], 8) == 0.0
    # brute force over the completion instants
    caps, M = [1.0, 0.75, 0.3, 0.9], 23
    cands = sorted(k / c for c in caps for k in range(1, M + 1))
    t_star = next(t for t in cands if sum(math.floor(t * c + 1e-9) for c in caps) >= M)
    assert integer_capacity(caps, M) == pytest.approx(M / t_star)


def test_one_gpu_loss_costs_resihp_less_than_dropping_a_replica():
    job = JobConfig(gpus=1024, tp=8, pp=16)
    thr = {}
    for p in [resihp_params(job), *baseline_params(job)]:
        st = ClusterState(job, p)
        st.fail([5], math.inf)
        st.refresh([5])
        thr[p.name] = st.throughput()
    assert thr["ResiHP"] > thr["torchft-bp"] and thr["ResiHP"] > thr["ReCycle"] - 1e-9
    assert thr["torchft"] == pytest.approx(7 / 8)


def test_simulation_accounting():
    job = JobConfig(gpus=1024, tp=8, pp=16, iteration_s=10.0)
    horizon = 86400.0
    for p in [ideal_params(), resihp_params(job), *baseline_params(job)]:
        assert simulate([], job, p, horizon).ettr == pytest.approx(1.0)
    events = [Event(4000.0, "fail", "gpu", "faulty_gpu", (17,), 7200.0)]
    res = {p.name: simulate(events, job, p, horizon) for p in [resihp_params(job), *baseline_params(job)]}
    assert res["ResiHP"].ettr > res["torchft-bp"].ettr > res["NVRx"].ettr
    assert res["NVRx"].lost_s > 0 and res["ResiHP"].lost_s <= job.iteration_s
    spared = simulate(events, JobConfig(gpus=1024, tp=8, pp=16, iteration_s=10.0, spare_nodes=1),
                      baseline_params(job)[1], horizon)
    assert spared.degraded_loss_s < res["torchft-bp"].degraded_loss_s
    slow = [Event(100.0, "slow", "gpu", "fail_slow", (3,), 5000.0, 2.0)]
    r = simulate(slow, job, resihp_params(job), horizon)
    assert 0.97 < r.ettr < 1.0 and r.events == 1  # detected after 3 iterations and migrated
