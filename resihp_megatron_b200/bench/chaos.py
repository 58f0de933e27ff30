"""Real-process chaos benchmark on CPU (8 gloo workers, TP2 x PP2 x DP2): MTTR breakdown.

Faults: ``kill`` (SIGKILL) and ``hang`` (SIGSTOP: alive, heartbeats and progress frozen) are
injected from outside the workers at a recorded time ``t0``; ``slow`` is a 2x fail-slow of one
rank's compute from the in-process injector (``slow@iter=...:factor=2``: each timed chunk is
stretched by a busy wait), found by the residual-BOCD detector service, with ``t0`` the moment
the coordinator sees the victim reach that iteration.  (A SIGSTOP/SIGCONT duty cycle is not used
for ``slow``: with sub-millisecond compute chunks it mostly stretches communication waits, which
the residual detector's predictor rightly does not read as a slower device.)  The
coordinator's transaction marks split recovery into detection, abort, planning, generation
build + state migration, and commit.  Each trial also checks that the survivors' losses and
final shards equal single-process training.  The CPU harness bounds the absolute numbers
(gloo, process start-up, Python); the breakdown is what carries over to GPUs.
(Reference: ``resihp/bench/chaos.py:84-186``.)
"""

from __future__ import annotations

import json
import os
import signal
import statistics
import sys
import tempfile
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
DEMO = str(ROOT / "examples" / "hetero_demo.py")
FAULTS = ("kill", "hang", "slow")
PHASES = ("detect", "abort", "plan", "build_migrate", "commit")


def _wait(pred, timeout: float, what: str) -> None:
    deadline = time.monotonic() + timeout
    while not pred():
        if time.monotonic() > deadline:
            raise TimeoutError(what)
        time.sleep(0.02)


def _progress(coord, worker_id: str) -> int:
    for w in coord.membership.alive():
        if w.worker_id == worker_id:
            return w.progress.get("iteration", -1)
    return -1


def verify(out: Path, world: list[str]) -> bool:
    from ..runtime.reference_model import RefModelConfig, reference_train
    from ..state.layer_registry import reference_specs
    from ..state.rng_data import IndexAddressableSampler

    infos = {w: json.loads((out / f"{w}.json").read_text()) for w in world if (out / f"{w}.json").exists()}
    iterations = 1 + max(int(i) for info in infos.values() for i in info["losses"])
    cfg = RefModelConfig()
    ref_losses, ref_params = reference_train(cfg, IndexAddressableSampler(256, 16, 2, seed=7), iterations)
    specs = reference_specs(cfg)
    for w, info in infos.items():
        if info.get("standby"):
            continue
        if any(abs(v - ref_losses[int(i)]) > 1e-9 * abs(ref_losses[int(i)]) for i, v in info["losses"].items()):
            return False
        shards = torch.load(out / f"{w}.pt")
        for key, iv in info["layout"].items():
            spec = specs[key]
            want = ref_params[key] if spec.dim is None else ref_params[key].narrow(spec.dim, iv[0], iv[1] - iv[0])
            if not torch.allclose(shards[key], want, rtol=1e-9, atol=1e-11):
                return False
    return True


def breakdown(history: list[dict], t0: float) -> dict:
    """Phase durations of the first transaction that followed the fault."""
    after = [h for h in history if h["t"] >= t0]
    fail = next((h for h in after if h["event"] == "failure" or h["event"] == "notice"), None)
    if fail is None:
        return {}
    gen = next(h["generation"] for h in after if h["event"] == "notice" and h["t"] >= fail["t"])
    mark = {h["event"]: h["t"] for h in after if h.get("generation") == gen}
    if "commit" not in mark:
        return {}
    steps = [t0, fail["t"], mark.get("aborted", fail["t"]), mark.get("planned", fail["t"]),
             mark.get("ready", mark["commit"]), mark["commit"]]
    out = {p: max(0.0, b - a) for p, a, b in zip(PHASES, steps, steps[1:])}
    out["total"] = mark["commit"] - t0
    return out


def run_trial(fault: str, iterations: int = 80, inject_after: int | None = None, iter_sleep: float = 0.05,
              slow_factor: float = 2.0) -> dict:
    from ..control.agent import NodeAgent
    from ..control.coordinator import Coordinator
    from ..detect.service import DetectorService
    from ..plan.coordinator_adapter import make_hetero_planner
    from ..train.demo_planners import HETERO_REF

    # the detector calibrates its noise prior during warm-up: start a slowdown after it
    inject_after = inject_after if inject_after is not None else (20 if fault == "slow" else 8)
    out = Path(tempfile.mkdtemp(prefix=f"resihp-chaos-{fault}-"))
    victim_id = "n0g0" if fault == "slow" else "n0g3"  # slow: a rank that reports its group's timings
    # gloo cannot abort an op blocked on a frozen peer, so the hang timeout must exceed the
    # communication timeout (10 s here) or the survivors' wait would look like a second hang
    coord = Coordinator(planner=make_hetero_planner(HETERO_REF), expected_workers=8, lease_timeout=2.0,
                        hang_timeout=30.0, abort_timeout=30.0, ready_timeout=120.0)
    svc = DetectorService(coord, warmup=6, min_increase=0.5) if fault == "slow" else None
    if svc is not None:
        coord.report_handler = svc.handle
    coord.start()
    env = {"PYTHONPATH": str(ROOT), "RESIHP_LOG_LEVEL": "ERROR", "OMP_NUM_THREADS": "1"}
    if fault == "slow":
        env["RESIHP_FAULTS"] = f"slow@iter={inject_after}:target={victim_id}:factor={slow_factor}"
    agents, stop = [], threading.Event()
    try:
        for n in range(2):
            ag = NodeAgent(f"n{n}", [coord.address], hb_interval=0.1, worker_timeout=3.0).start()
            ag.spawn([sys.executable, DEMO, "--iterations", str(iterations), "--out", str(out), "--timeout", "10",
                      "--iter-sleep", str(iter_sleep)], 4, env=env)
            agents.append(ag)
        _wait(lambda: coord.committed_generation >= 1, 60, "start")
        victim = agents[0].workers[victim_id].proc.pid
        if fault == "slow":
            _wait(lambda: _progress(coord, victim_id) >= inject_after, 120, "warm-up")
            t0 = time.monotonic()
        else:
            _wait(lambda: min((w.progress.get("iteration", -1) for w in coord.membership.alive()), default=-1)
                  >= inject_after, 120, "warm-up")
            t0 = time.monotonic()
            os.kill(victim, signal.SIGKILL if fault == "kill" else signal.SIGSTOP)
        _wait(lambda: coord.committed_generation >= 2, 240, "recovery commit")
        stop.set()
        procs = [w.proc for ag in agents for w in ag.workers.values()]
        _wait(lambda: all(p.poll() is not None for p in procs if p.pid != victim) or coord.phase == "finished",
              600, "job end")
        _wait(lambda: all(p.poll() is not None for p in procs if p.pid != victim), 60, "workers to exit")
        res = {"fault": fault, "breakdown": breakdown(coord.history, t0), "world": list(coord.world),
               "exact": verify(out, list(coord.world)),
               "reason": next((h.get("reason") for h in coord.history if h["event"] == "commit" and h["t"] >= t0),
                              None)}
        return res
    finally:
        stop.set()
        for ag in agents:
            ag.stop(kill_workers=True)
        coord.stop()


def run(trials: int = 3, faults=FAULTS) -> dict:
    out: dict = {"trials": {}, "summary": {}}
    for f in faults:
        rows = [run_trial(f) for _ in range(trials)]
        out["trials"][f] = rows
        ok = [r for r in rows if r["breakdown"]]
        out["summary"][f] = {k: statistics.fmean(r["breakdown"][k] for r in ok) for k in (*PHASES, "total")} if ok \
            else {}
        out["summary"][f]["exact"] = all(r["exact"] for r in rows)
    return out


def to_markdown(res: dict) -> str:
    lines = ["| fault | detect (s) | abort | plan | build + migrate | commit | total MTTR | exact |",
             "|---|---|---|---|---|---|---|---|"]
    for f, s in res["summary"].items():
        if "total" not in s:
            lines.append(f"| {f} | - | - | - | - | - | - | {s.get('exact')} |")
            continue
        lines.append(f"| {f} | " + " | ".join(f"{s[k]:.2f}" for k in (*PHASES, "total")) + f" | {s['exact']} |")
    return "\n".join(lines)
