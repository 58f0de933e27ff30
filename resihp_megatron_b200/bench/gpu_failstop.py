"""Fail-stop recovery on GPUs through the control plane, timed from the fault to the commit.

A coordinator and one node agent start ``examples/gpu_hybrid_demo.py`` on ``n`` GPUs of this node
(TP x PP x DP from ``layout_for(n)``, sequence parallel, NCCL collectives with NVLS off).  One
worker SIGKILLs itself at an iteration boundary after a device synchronise (so it leaves with no
kernel or collective in flight) and stamps the instant on the machine-wide monotonic clock.  The
survivors learn of it from the coordinator, abort the generation's communicators, take the
re-planned layout, migrate parameter and Adam slices and replay the interrupted iteration.  The
coordinator's transaction marks split the recovery into detect / abort / plan / build + migrate /
commit.  Every failure is made on the host; no kernel faults, traps or hangs.
(Reference: ``resihp/bench/chaos.py:84-186`` on CPU workers; here the workers run the GPU runtime.)
"""

from __future__ import annotations

import json
import os
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
DEMO = ROOT / "examples" / "gpu_hybrid_demo.py"


def layout_for(n: int) -> tuple[int, int, int]:
    """(tp, pp, dp) of the demo job on ``n`` GPUs: benchmark config 2's TP2 x PP2 x DP2 at 8,
    scaled down with a data-parallel replica kept (the killed rank's slices need a holder)."""
    return {2: (1, 1, 2), 4: (2, 1, 2), 8: (2, 2, 2)}.get(n, (1, 1, n))


def run_trial(n: int, iterations: int = 6, kill_iteration: int = 2, out: str | None = None,
              deadline_s: float = 600.0) -> dict:
    """Run the job, kill its last worker after ``kill_iteration`` committed; returns the exit
    codes, the phase breakdown and every survivor's per-iteration losses."""
    from ..control.agent import NodeAgent
    from ..control.coordinator import Coordinator
    from ..plan.coordinator_adapter import make_hetero_planner
    from ..train.demo_planners import gpu_planner_config
    from .chaos import breakdown

    tp, pp, dp = layout_for(n)
    victim = f"n0g{n - 1}"
    outdir = Path(out or tempfile.mkdtemp(prefix="resihp-gpu-failstop-"))
    outdir.mkdir(parents=True, exist_ok=True)
    stamp = outdir / "fault_stamp.txt"
    env = {"RESIHP_FAULTS": f"kill@iter={kill_iteration}:target={victim}:phase=boundary",
           "RESIHP_FAULT_STAMP": str(stamp), "PYTHONPATH": str(ROOT), "OMP_NUM_THREADS": "1",
           "NCCL_NVLS_ENABLE": "0", "RESIHP_LOG_LEVEL": "WARNING"}
    coord = Coordinator(planner=make_hetero_planner(gpu_planner_config(tp=tp, pp=pp, dp=dp)), expected_workers=n,
                        lease_timeout=3.0, hang_timeout=120.0, abort_timeout=60.0, ready_timeout=240.0).start()
    cmd = [sys.executable, str(DEMO), "--iterations", str(iterations), "--out", str(outdir), "--timeout", "20",
           "--device", "cuda", "--tp-impl", "collective"]
    agent = None
    try:
        agent = NodeAgent("n0", [coord.address], hb_interval=0.1, worker_timeout=5.0).start()
        # the demo workers join the coordinator's job, not a launcher's (e.g. torchrun's) group
        launcher = {k: os.environ.pop(k) for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE",
                                                   "GROUP_RANK", "MASTER_ADDR", "MASTER_PORT") if k in os.environ}
        try:
            agent.spawn(cmd, n, env=env)
        finally:
            os.environ.update(launcher)
        end = time.monotonic() + deadline_s
        while time.monotonic() < end:
            if all(w.proc.poll() is not None for w in agent.workers.values()):
                break
            time.sleep(0.5)
        codes = {w.worker_id: w.proc.returncode for w in agent.workers.values()}
        history = list(coord.history)
    finally:
        if agent is not None:
            agent.stop(kill_workers=True)
        coord.stop()
    phases, events = None, None
    if stamp.exists():
        t_fault = float(stamp.read_text().split()[1])
        phases = breakdown(history, t_fault)
        # the coordinator's transaction events, seconds after the fault (machine-wide monotonic clock)
        events = [(h["event"], round(h["t"] - t_fault, 4)) for h in history if h["t"] >= t_fault][:16]
    losses, rebuild = {}, {}
    for w in codes:
        f = outdir / f"{w}.json"
        if w != victim and f.exists():
            info = json.loads(f.read_text())
            if not info["standby"]:
                losses[w] = {int(k): v for k, v in info["losses"].items()}
                steps = dict(info.get("build_steps_s") or {})
                if stamp.exists():  # absolute instants -> seconds after the fault
                    t_fault = float(stamp.read_text().split()[1])
                    steps = {k: (round(v - t_fault, 4) if k.endswith("_at") else v) for k, v in steps.items()}
                rebuild[w] = dict(info.get("last_recovery") or {}, worker_steps_s=steps)
    return {"gpus": n, "layout": f"tp{tp}pp{pp}dp{dp}", "victim": victim, "codes": codes, "phases_s": phases,
            "events_s": events,
            "losses": losses, "rebuild_s": rebuild, "out": str(outdir)}


def main(argv=None) -> None:
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=2)
    ap.add_argument("--iterations", type=int, default=6)
    args = ap.parse_args(argv)
    print(json.dumps(run_trial(args.gpus, args.iterations)), flush=True)


if __name__ == "__main__":
    main()
