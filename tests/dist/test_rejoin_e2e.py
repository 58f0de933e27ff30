"""Rejoin end to end on CPU worker processes: a TP2 x PP2 x DP2 job starts on 7 workers (the
planner gives one group TP1), a replacement worker registers mid-run, the coordinator re-plans
with it (the group grows back to TP2), the newcomer receives its parameter and Adam slices from
the running workers, and every worker's losses and final shards equal single-process training."""

import sys
import time
from pathlib import Path

import pytest

pytestmark = [pytest.mark.dist, pytest.mark.slow]

ROOT = Path(__file__).resolve().parents[2]


def test_replacement_worker_joins_and_receives_its_state(tmp_path):
    from resihp_megatron_b200.bench.chaos import verify
    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator
    from resihp_megatron_b200.plan.coordinator_adapter import make_hetero_planner
    from resihp_megatron_b200.train.demo_planners import HETERO_REF

    coord = Coordinator(planner=make_hetero_planner(HETERO_REF), expected_workers=7, lease_timeout=3.0,
                        hang_timeout=60.0, abort_timeout=30.0, ready_timeout=120.0).start()
    env = {"PYTHONPATH": str(ROOT), "OMP_NUM_THREADS": "1", "RESIHP_LOG_LEVEL": "ERROR"}
    cmd = [sys.executable, str(ROOT / "examples" / "hetero_demo.py"), "--iterations", "30", "--out", str(tmp_path),
           "--timeout", "20", "--iter-sleep", "0.25"]
    agents = []
    try:
        for n, k in ((0, 4), (1, 3)):
            ag = NodeAgent(f"n{n}", [coord.address], hb_interval=0.1, worker_timeout=5.0).start()
            ag.spawn(cmd, k, env=env)
            agents.append(ag)
        deadline = time.monotonic() + 120
        while time.monotonic() < deadline and coord.committed_generation < 1:
            time.sleep(0.1)
        assert coord.committed_generation == 1 and len(coord.world) == 7
        agents[1].spawn(cmd, 1, env=env, first_rank=3)  # the replacement: n1g3
        deadline = time.monotonic() + 300
        while time.monotonic() < deadline:
            if all(w.proc.poll() is not None for ag in agents for w in ag.workers.values()):
                break
            time.sleep(0.5)
        codes = {w.worker_id: w.proc.returncode for ag in agents for w in ag.workers.values()}
        joined = [h for h in coord.history if h["event"] == "commit" and str(h.get("reason", "")).startswith("join")]
    finally:
        for ag in agents:
            ag.stop(kill_workers=True)
        coord.stop()
    assert all(c == 0 for c in codes.values()), codes
    assert joined, coord.history
    assert "n1g3" in coord.world and len(coord.world) == 8
    assert verify(tmp_path, sorted(codes))
