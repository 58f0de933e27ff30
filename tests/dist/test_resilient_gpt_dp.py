"""benchmark config 1 end to end: 8 CPU workers on 2 simulated nodes train the float64 GPT with
replica DP; ``kill -9`` of n0g3 in the forward pass of iteration 3; the 7 survivors re-plan,
roll back / forward, and finish 20 iterations.  Every survivor's loss trajectory must be
bitwise equal to single-process training."""

import json
import os
import sys
import time
from pathlib import Path

import pytest

pytestmark = [pytest.mark.dist, pytest.mark.slow]

ROOT = Path(__file__).resolve().parents[2]


def _run_job(tmp_path, faults: str, iterations: int):
    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator
    from resihp_megatron_b200.plan.dp_planner import make_dp_planner

    coord = Coordinator(planner=make_dp_planner(8), expected_workers=8, hang_timeout=60, lease_timeout=5).start()
    agents = []
    env = {"RESIHP_FAULTS": faults, "PYTHONPATH": str(ROOT), "OMP_NUM_THREADS": "1"}
    cmd = [sys.executable, str(ROOT / "examples" / "gpt_dp_demo.py"), "--iterations", str(iterations),
           "--out", str(tmp_path)]
    try:
        for n in range(2):
            ag = NodeAgent(f"n{n}", [coord.address]).start()
            ag.spawn(cmd, 4, env=env, devices=["cpu"] * 4)
            agents.append(ag)
        deadline = time.monotonic() + 400
        while time.monotonic() < deadline:
            if all(w.proc.poll() is not None for ag in agents for w in ag.workers.values()):
                break
            time.sleep(0.5)
        codes = {w.worker_id: w.proc.returncode for ag in agents for w in ag.workers.values()}
        return codes, coord.history
    finally:
        for ag in agents:
            ag.stop(kill_workers=True)
        coord.stop()


def test_kill9_recovery_is_bit_identical(tmp_path):
    from resihp_megatron_b200.runtime.reference_gpt import GPTRefConfig, train_single_process

    iterations = 20
    codes, history = _run_job(tmp_path, "kill@iter=3:target=n0g3:phase=forward", iterations)
    assert codes["n0g3"] == -9, codes
    survivors = [w for w in codes if w != "n0g3"]
    assert all(codes[w] == 0 for w in survivors), codes
    ref_losses, ref_params = train_single_process(GPTRefConfig(), iterations)
    import torch

    for w in survivors:
        res = json.loads((tmp_path / f"{w}.json").read_text())
        losses = [res["losses"][str(i)] for i in range(iterations)]
        assert losses == ref_losses, (w, losses[:5], ref_losses[:5])  # bitwise, not approximate
        params = torch.load(tmp_path / f"{w}.pt")
        for k, v in ref_params.items():
            assert torch.equal(params[k], v), (w, k)
    commits = [h for h in history if h["event"] == "commit"]
    assert len(commits) >= 2 and len(commits[-1]["world"]) == 7
