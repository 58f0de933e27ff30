"""Fail-slow detection accuracy on packed variable-length data (the setting of ResiHP Table 5).

Four detectors -- Greyhound-style raw series, ResiHP as published (raw series plus the
predicted-time filter), the residual series, and the per-(replica, stage) service view -- run on
synthetic traces with long-document bursts, healthy and with an injected slowdown of several
factors.  Reported per detector: validations on healthy traces (false alarms), detections within
``horizon`` iterations of the onset, false alarms before it, mean latency and (service view)
whether the slow group was the one flagged.
Parity: ``resihp/bench/detection.py:1-55`` (same experiment and table).
"""

from __future__ import annotations

import statistics
from collections import Counter

from ..detect.synthetic import SyntheticJob, evaluate_detector, generate_trace

MODES = ("greyhound", "paper", "residual", "group")


def _score(result: dict, slow_at: int, horizon: int, mode: str, tally: dict) -> None:
    found = result["detections"]
    tally["false_alarms"] += sum(d < slow_at for d in found)
    in_time = [i for i, d in enumerate(found) if slow_at <= d <= slow_at + horizon]
    if not in_time:
        return
    first = in_time[0]
    tally["detected"] += 1
    tally["latency"].append(found[first] - slow_at)
    if mode == "group":
        tally["localized"] += int(result["groups"][first] == [(0, 1)])


def run(seeds: int = 20, iterations: int = 120, slow_at: int = 70, factors=(1.3, 1.6, 2.0), horizon: int = 10) -> dict:
    job = SyntheticJob()
    healthy = Counter({m: 0 for m in MODES})
    for s in range(seeds):
        trace = generate_trace(job, iterations, seed=1000 + s)
        for m in MODES:
            healthy[m] += evaluate_detector(job, trace, m)["validations"]
    slow = {}
    for f in factors:
        tallies = {m: dict(detected=0, false_alarms=0, latency=[], localized=0) for m in MODES}
        for s in range(seeds):
            trace = generate_trace(job, iterations, seed=2000 + s, slow_at=slow_at, factor=f)
            for m in MODES:
                _score(evaluate_detector(job, trace, m), slow_at, horizon, m, tallies[m])
        slow[str(f)] = tallies
    return {"healthy": dict(healthy), "slow": slow, "seeds": seeds, "slow_at": slow_at, "horizon": horizon}


def to_markdown(res: dict) -> str:
    header = ("| detector | validations on healthy traces | slowdown | detected | false alarms before onset | "
              "mean latency (iterations) | localized |")
    rows = [header, "|---|---|---|---|---|---|---|"]
    for factor, tallies in res["slow"].items():
        for m in MODES:
            t = tallies[m]
            latency = f"{statistics.fmean(t['latency']):.1f}" if t["latency"] else "-"
            localized = f"{t['localized']}/{t['detected']}" if m == "group" else "n/a"
            rows.append(f"| {m} | {res['healthy'][m]} | {factor}x | {t['detected']}/{res['seeds']} | "
                        f"{t['false_alarms']} | {latency} | {localized} |")
    return "\n".join(rows)
