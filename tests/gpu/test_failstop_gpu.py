"""Fail-stop recovery on GPUs through the control plane (needs 2 or more GPUs).

A coordinator and one node agent run ``examples/gpu_hybrid_demo.py`` on N = 2 or 4 GPUs
(TP1 x DP2 or TP2 x DP2, sequence parallel, NCCL collectives, NVLS off).  One worker SIGKILLs
itself at an iteration boundary, after a device synchronise, so it leaves with nothing in flight;
the survivors learn of it from the coordinator, abort the generation's communicators, take the
re-planned layout, migrate parameter and Adam slices peer to peer and replay the interrupted
iteration.  Checks: every survivor finishes with a loss for every iteration, the losses follow a
one-GPU run of the same model on the same global batches (bf16 rounding of the collectives
aside), and the fault->commit phases are reported (on the machine-wide monotonic clock, from the
victim's own stamp).  Failures are made on the host only: no kernel faults, traps or hangs."""

import json
import os
import subprocess
import sys
import time
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[2]
ITERS = 6

REFERENCE = """
import json, sys
import torch
from resihp_megatron_b200.train.demo_planners import GPU_DEMO, GPU_DEMO_MICRO
from resihp_megatron_b200.train.hybrid_trainer import GPUHybridTrainer, ensure_process_group
torch.cuda.set_device(0)
ensure_process_group(torch.device("cuda", 0))
tr = GPUHybridTrainer(GPU_DEMO, tp=1, pp=1, dp=1, global_batch=GPU_DEMO_MICRO, micro_batch=1, seq_len=GPU_DEMO.seq_len,
                      tp_impl="collective", dp_impl="collective", device="cuda:0", lr=1e-2)
losses = [float(tr.train_step()) for _ in range(int(sys.argv[1]))]
tr.close()
print(json.dumps(losses))
"""


def _layout(n: int) -> tuple[int, int, int]:
    return (1, 1, 2) if n == 2 else (2, 1, 2)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
def test_kill_at_boundary_recovers_on_gpus(tmp_path):
    from resihp_megatron_b200.bench.chaos import breakdown
    from resihp_megatron_b200.control.agent import NodeAgent
    from resihp_megatron_b200.control.coordinator import Coordinator
    from resihp_megatron_b200.plan.coordinator_adapter import make_hetero_planner
    from resihp_megatron_b200.train.demo_planners import gpu_planner_config

    n = 4 if torch.cuda.device_count() >= 4 else 2
    tp, pp, dp = _layout(n)
    victim = f"n0g{n - 1}"
    stamp = tmp_path / "fault_stamp.txt"
    env = {"RESIHP_FAULTS": f"kill@iter=2:target={victim}:phase=boundary", "RESIHP_FAULT_STAMP": str(stamp),
           "PYTHONPATH": str(ROOT), "OMP_NUM_THREADS": "1", "NCCL_NVLS_ENABLE": "0", "RESIHP_LOG_LEVEL": "WARNING"}
    coord = Coordinator(planner=make_hetero_planner(gpu_planner_config(tp=tp, pp=pp, dp=dp)), expected_workers=n,
                        lease_timeout=3.0, hang_timeout=120.0, abort_timeout=60.0, ready_timeout=240.0).start()
    cmd = [sys.executable, str(ROOT / "examples" / "gpu_hybrid_demo.py"), "--iterations", str(ITERS), "--out",
           str(tmp_path), "--timeout", "20", "--device", "cuda", "--tp-impl", "collective"]
    agent = None
    try:
        agent = NodeAgent("n0", [coord.address], hb_interval=0.1, worker_timeout=5.0).start()
        agent.spawn(cmd, n, env=env)
        deadline = time.monotonic() + 600
        while time.monotonic() < deadline:
            if all(w.proc.poll() is not None for w in agent.workers.values()):
                break
            time.sleep(0.5)
        codes = {w.worker_id: w.proc.returncode for w in agent.workers.values()}
        history = list(coord.history)
    finally:
        if agent is not None:
            agent.stop(kill_workers=True)
        coord.stop()
    assert codes[victim] == -9, codes
    survivors = [w for w in codes if w != victim]
    assert all(codes[w] == 0 for w in survivors), codes

    t0 = float(stamp.read_text().split()[1])
    phases = breakdown(history, t0)
    print(json.dumps({"gpus": n, "layout": f"tp{tp}pp{pp}dp{dp}", "fault_to_commit_s": phases}))
    assert phases and phases["total"] > 0

    ref = subprocess.run([sys.executable, "-c", REFERENCE, str(ITERS)], cwd=ROOT, capture_output=True, text=True,
                         timeout=600, env=dict(os.environ, PYTHONPATH=str(ROOT)))
    assert ref.returncode == 0, ref.stderr[-2000:]
    want = json.loads(ref.stdout.strip().splitlines()[-1])
    trained = 0
    for w in survivors:
        info = json.loads((tmp_path / f"{w}.json").read_text())
        if info["standby"]:
            continue
        trained += 1
        assert len(info["generations"]) >= 2, info
        assert sorted(int(k) for k in info["losses"]) == list(range(ITERS)), info["losses"]
        for it, v in info["losses"].items():
            assert abs(v - want[int(it)]) <= 2e-2 * abs(want[int(it)]), (w, it, v, want)
    assert trained >= 1
