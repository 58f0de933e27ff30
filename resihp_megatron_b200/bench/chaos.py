"""Real-process chaos benchmark on the CPU (8 gloo workers, TP2 x PP2 x DP2): MTTR breakdown.

Faults: ``kill`` (SIGKILL) and ``hang`` (SIGSTOP: alive, with heartbeats and progress frozen) are
injected from outside the workers at a recorded instant ``t0``; ``slow`` is a 2x fail-slow of
one rank's compute from the in-process injector (``slow@iter=...:factor=2``: each timed chunk is
stretched by a busy wait), found by the residual-BOCD detector service, with ``t0`` the moment
the coordinator sees the victim reach that iteration.  (A SIGSTOP / SIGCONT duty cycle is not
used for ``slow``: with sub-millisecond compute chunks it mostly stretches communication waits,
which the residual detector's predictor rightly does not read as a slower device.)  The
coordinator's transaction marks split a recovery into detection, abort, planning, generation
build with state migration, and commit.  Every trial also checks that the survivors' losses and
final shards equal single-process training.  The CPU harness bounds the absolute numbers (gloo,
process start-up, Python); the breakdown is what carries over to GPUs.
Parity: ``resihp/bench/chaos.py:84-186`` (same faults, phases and exactness check).
"""

from __future__ import annotations

import json
import os
import signal
import statistics
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
DEMO = str(ROOT / "examples" / "hetero_demo.py")
FAULTS = ("kill", "hang", "slow")
PHASES = ("detect", "abort", "plan", "build_migrate", "commit")


def _until(condition, timeout: float, what: str) -> None:
    give_up = time.monotonic() + timeout
    while not condition():
        if time.monotonic() > give_up:
            raise TimeoutError(what)
        time.sleep(0.02)


def _iteration_of(coord, worker_id: str) -> int:
    rec = next((w for w in coord.membership.alive() if w.worker_id == worker_id), None)
    return -1 if rec is None else rec.progress.get("iteration", -1)


def _slowest_iteration(coord) -> int:
    return min((w.progress.get("iteration", -1) for w in coord.membership.alive()), default=-1)


def verify(out: Path, world: list[str]) -> bool:
    """Every survivor's losses (rtol 1e-9) and final shards equal single-process training."""
    from ..runtime.reference_model import RefModelConfig, reference_train
    from ..state.layer_registry import reference_specs
    from ..state.rng_data import IndexAddressableSampler

    reports = {w: json.loads((out / f"{w}.json").read_text()) for w in world if (out / f"{w}.json").exists()}
    steps = 1 + max(int(i) for r in reports.values() for i in r["losses"])
    cfg = RefModelConfig()
    want_losses, want_params = reference_train(cfg, IndexAddressableSampler(256, 16, 2, seed=7), steps)
    specs = reference_specs(cfg)
    for worker, report in reports.items():
        if report.get("standby"):
            continue
        for it, loss in report["losses"].items():
            if abs(loss - want_losses[int(it)]) > 1e-9 * abs(want_losses[int(it)]):
                return False
        shards = torch.load(out / f"{worker}.pt")
        for key, (lo, hi) in report["layout"].items():
            spec = specs[key]
            full = want_params[key]
            expected = full if spec.dim is None else full.narrow(spec.dim, lo, hi - lo)
            if not torch.allclose(shards[key], expected, rtol=1e-9, atol=1e-11):
                return False
    return True


def breakdown(history: list[dict], t0: float) -> dict:
    """Phase durations of the first transaction after the fault (empty if it never committed)."""
    later = [h for h in history if h["t"] >= t0]
    first = next((h for h in later if h["event"] in ("failure", "notice")), None)
    if first is None:
        return {}
    gen = next(h["generation"] for h in later if h["event"] == "notice" and h["t"] >= first["t"])
    at = {h["event"]: h["t"] for h in later if h.get("generation") == gen}
    if "commit" not in at:
        return {}
    edges = [t0, first["t"], at.get("aborted", first["t"]), at.get("planned", first["t"]),
             at.get("ready", at["commit"]), at["commit"]]
    phases = {name: max(0.0, end - start) for name, start, end in zip(PHASES, edges, edges[1:])}
    phases["total"] = at["commit"] - t0
    return phases


class _Trial:
    """Coordinator, two simulated nodes of four workers, one fault, one recovery."""

    def __init__(self, fault: str, iterations: int, inject_after: int, iter_sleep: float, slow_factor: float):
        self.fault, self.iterations, self.inject_after = fault, iterations, inject_after
        self.iter_sleep, self.slow_factor = iter_sleep, slow_factor
        self.out = Path(tempfile.mkdtemp(prefix=f"resihp-chaos-{fault}-"))
        self.victim_id = "n0g0" if fault == "slow" else "n0g3"  # slow: a rank that reports its group's timings
        self.coord, self.agents = None, []

    def start(self) -> None:
        from ..control.agent import NodeAgent
        from ..control.coordinator import Coordinator
        from ..detect.service import DetectorService
        from ..plan.coordinator_adapter import make_hetero_planner
        from ..train.demo_planners import HETERO_REF

        # gloo cannot abort an op blocked on a frozen peer, so the hang timeout must exceed the
        # communication timeout (10 s) or the survivors' wait would look like a second hang
        self.coord = Coordinator(planner=make_hetero_planner(HETERO_REF), expected_workers=8, lease_timeout=2.0,
                                 hang_timeout=30.0, abort_timeout=30.0, ready_timeout=120.0)
        if self.fault == "slow":
            self.coord.report_handler = DetectorService(self.coord, warmup=6, min_increase=0.5).handle
        self.coord.start()
        env = {"PYTHONPATH": str(ROOT), "RESIHP_LOG_LEVEL": "ERROR", "OMP_NUM_THREADS": "1"}
        if self.fault == "slow":
            env["RESIHP_FAULTS"] = f"slow@iter={self.inject_after}:target={self.victim_id}:factor={self.slow_factor}"
        cmd = [sys.executable, DEMO, "--iterations", str(self.iterations), "--out", str(self.out), "--timeout", "10",
               "--iter-sleep", str(self.iter_sleep)]
        for n in range(2):
            agent = NodeAgent(f"n{n}", [self.coord.address], hb_interval=0.1, worker_timeout=3.0).start()
            agent.spawn(cmd, 4, env=env)
            self.agents.append(agent)

    def inject(self) -> float:
        """Wait for the warm-up, inject, return the fault instant."""
        coord = self.coord
        _until(lambda: coord.committed_generation >= 1, 60, "start")
        if self.fault == "slow":  # the injector fires itself at iteration ``inject_after``
            _until(lambda: _iteration_of(coord, self.victim_id) >= self.inject_after, 120, "warm-up")
            return time.monotonic()
        _until(lambda: _slowest_iteration(coord) >= self.inject_after, 120, "warm-up")
        t0 = time.monotonic()
        os.kill(self.victim_pid, signal.SIGKILL if self.fault == "kill" else signal.SIGSTOP)
        return t0

    @property
    def victim_pid(self) -> int:
        return self.agents[0].workers[self.victim_id].proc.pid

    def finish(self, t0: float) -> dict:
        coord = self.coord
        _until(lambda: coord.committed_generation >= 2, 240, "recovery commit")
        others = [w.proc for a in self.agents for w in a.workers.values() if w.proc.pid != self.victim_pid]
        _until(lambda: all(p.poll() is not None for p in others) or coord.phase == "finished", 600, "job end")
        _until(lambda: all(p.poll() is not None for p in others), 60, "workers to exit")
        reason = next((h.get("reason") for h in coord.history if h["event"] == "commit" and h["t"] >= t0), None)
        return {"fault": self.fault, "breakdown": breakdown(coord.history, t0), "world": list(coord.world),
                "exact": verify(self.out, list(coord.world)), "reason": reason}

    def close(self) -> None:
        for agent in self.agents:
            agent.stop(kill_workers=True)
        if self.coord is not None:
            self.coord.stop()


def run_trial(fault: str, iterations: int = 80, inject_after: int | None = None, iter_sleep: float = 0.05,
              slow_factor: float = 2.0) -> dict:
    # the detector calibrates its noise prior during its warm-up: a slowdown starts after it
    after = inject_after if inject_after is not None else (20 if fault == "slow" else 8)
    trial = _Trial(fault, iterations, after, iter_sleep, slow_factor)
    try:
        trial.start()
        return trial.finish(trial.inject())
    finally:
        trial.close()


def run(trials: int = 3, faults=FAULTS) -> dict:
    result: dict = {"trials": {}, "summary": {}}
    for fault in faults:
        rows = result["trials"][fault] = [run_trial(fault) for _ in range(trials)]
        timed = [r["breakdown"] for r in rows if r["breakdown"]]
        summary = {k: statistics.fmean(b[k] for b in timed) for k in (*PHASES, "total")} if timed else {}
        summary["exact"] = all(r["exact"] for r in rows)
        result["summary"][fault] = summary
    return result


def to_markdown(res: dict) -> str:
    table = ["| fault | detect (s) | abort | plan | build + migrate | commit | total MTTR | exact |",
             "|---|---|---|---|---|---|---|---|"]
    for fault, s in res["summary"].items():
        cells = [f"{s[k]:.2f}" for k in (*PHASES, "total")] if "total" in s else ["-"] * (len(PHASES) + 1)
        table.append(f"| {fault} | " + " | ".join(cells) + f" | {s.get('exact')} |")
    return "\n".join(table)


def main(argv=None) -> None:
    """One trial, printed as one JSON line (what ``bench.py`` reads for its fault->commit key)."""
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--fault", choices=FAULTS, default="kill")
    ap.add_argument("--iterations", type=int, default=40)
    args = ap.parse_args(argv)
    print(json.dumps(run_trial(args.fault, iterations=args.iterations)), flush=True)


if __name__ == "__main__":
    main()
