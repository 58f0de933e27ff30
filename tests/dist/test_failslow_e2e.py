"""Fail-slow end to end on CPU worker processes: one rank of a TP2 x PP2 x DP2 job computes 2x
slower from iteration 20 (in-process injector); the residual-BOCD detector service flags its
group from the timing reports, the coordinator re-plans around it (work shed by the planner),
and the run stays equal to single-process training."""

import pytest

pytestmark = [pytest.mark.dist, pytest.mark.slow]


def test_slow_rank_is_detected_and_the_plan_sheds_its_work():
    from resihp_megatron_b200.bench.chaos import run_trial

    r = run_trial("slow")
    assert r["reason"] and r["reason"].startswith("failslow:") and "n0g0" in r["reason"], r
    assert r["exact"], r
    assert r["breakdown"]["detect"] < 30.0, r
