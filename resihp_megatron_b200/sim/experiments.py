"""Cluster-scale experiments: ETTR across scales and policies, the loss breakdown, sensitivity.

The job is a 405B-class dense model on TP8 x PP16 (128 GPUs per replica) with 16 micro-batches
per replica, on the Llama 3 failure trace scaled to the cluster size.
Parity: ``resihp/sim/experiments.py:20-100`` (same job, sweeps and tables).
"""

from __future__ import annotations

import statistics
from collections import defaultdict

from .calibrate import PROFILE
from .cluster import JobConfig, baseline_params, ideal_params, resihp_params, simulate
from .traces import TraceConfig, generate, summarize

DEFAULT_SCALES = (1024, 4096, 16384, 32768, 65536)


def job_for(gpus: int, **kw) -> JobConfig:
    return JobConfig(gpus=gpus, tp=8, pp=16, iteration_s=10.0, microbatches_per_replica=16, min_tp=4,
                     tp_degrees=(1, 2, 4, 8), profile=PROFILE, **kw)


def policies(job: JobConfig, calib: dict, *, restart_s: float = 300.0, checkpoint_interval_s: float = 1200.0):
    baselines = baseline_params(job, restart_s=restart_s, checkpoint_interval_s=checkpoint_interval_s)
    return [ideal_params(), resihp_params(job, beta=calib["beta"], overhead=calib["overhead"]), *baselines]


def _mean_row(rows: list[dict]) -> dict:
    numeric = [k for k, v in rows[0].items() if isinstance(v, (int, float))]
    mean = {k: statistics.fmean(r[k] for r in rows) for k in numeric}
    mean["ettr_std"] = statistics.pstdev(r["ettr"] for r in rows)
    return mean


def run_cell(gpus: int, days: float, seeds: int, calib: dict, trace_kw=None, policy_kw=None,
             spare_frac: float = 0.0) -> dict:
    """Every policy on ``seeds`` traces of one cluster size; per-policy means over the seeds."""
    job = job_for(gpus, spare_nodes=int(round(spare_frac * gpus / 8)))
    rows: dict[str, list[dict]] = defaultdict(list)
    summaries = []
    for seed in range(seeds):
        cfg = TraceConfig(gpus=gpus, days=days, seed=seed, **(trace_kw or {}))
        events = generate(cfg)
        summaries.append(summarize(events, cfg))
        for policy in policies(job, calib, **(policy_kw or {})):
            rows[policy.name].append(simulate(events, job, policy, 86400.0 * days).to_json())
    return {"gpus": gpus, "days": days, "seeds": seeds, "trace": summaries[0] if summaries else {},
            "fail_stop_mean": statistics.fmean(s["fail_stop"] for s in summaries),
            "policies": {name: _mean_row(r) for name, r in rows.items()}}


def scale_sweep(calib: dict, scales=DEFAULT_SCALES, days: float = 30.0, seeds: int = 5) -> list[dict]:
    return [run_cell(gpus, days, seeds, calib) for gpus in scales]


def sensitivity(calib: dict, gpus: int = 16384, days: float = 30.0, seeds: int = 3) -> dict:
    """ETTR per policy while one assumption moves: restart time, GPU repair time, failure rate,
    fail-slow rate."""
    base = TraceConfig(gpus=gpus)

    def cell(**kw):
        return run_cell(gpus, days, seeds, calib, **kw)["policies"]

    knobs = {
        "restart_s": {str(int(r)): dict(policy_kw={"restart_s": r}) for r in (300.0, 600.0, 1200.0, 1800.0)},
        "gpu_repair_h": {str(int(h)): dict(trace_kw={"repair_median_s": dict(base.repair_median_s, gpu=h * 3600.0)})
                         for h in (6.0, 24.0, 72.0)},
        "fail_rate_x": {str(x): dict(trace_kw={"rate_scale": x}) for x in (0.5, 1.0, 2.0, 4.0)},
        "slow_rate_x": {str(x): dict(trace_kw={"slow_per_gpu_day": base.slow_per_gpu_day * x}) for x in (0.0, 1.0, 4.0)},
    }
    return {knob: {label: cell(**kw) for label, kw in settings.items()} for knob, settings in knobs.items()}


def scale_table(cells: list[dict]) -> str:
    names = list(cells[0]["policies"])
    rows = ["| policy | " + " | ".join(f"{c['gpus']:,} GPUs" for c in cells) + " |", "|---|" + "---|" * len(cells)]
    rows += [f"| {n} | " + " | ".join(f"{c['policies'][n]['ettr'] * 100:.1f}%" for c in cells) + " |" for n in names]
    rows.append("| fail-stop events | " + " | ".join(f"{c['fail_stop_mean']:.0f}" for c in cells) + " |")
    return "\n".join(rows)


def breakdown_table(cell: dict) -> str:
    rows = [f"| policy ({cell['gpus']:,} GPUs, {cell['days']:.0f} days) | ETTR | downtime | rollback | "
            "degraded throughput | mean MTTR (s) | p99 MTTR (s) |", "|---|---|---|---|---|---|---|"]
    for name, a in cell["policies"].items():
        pct = [f"{a[k] * 100:.2f}%" for k in ("ettr", "downtime_frac", "lost_frac", "degraded_frac")]
        rows.append(f"| {name} | " + " | ".join(pct) + f" | {a['mttr_mean_s']:.0f} | {a['mttr_p99_s']:.0f} |")
    return "\n".join(rows)


def sensitivity_table(sens: dict) -> str:
    lines = []
    for knob, cells in sens.items():
        names = list(next(iter(cells.values())))
        lines += [f"\n**{knob}**\n", "| policy | " + " | ".join(cells) + " |", "|---|" + "---|" * len(cells)]
        lines += [f"| {n} | " + " | ".join(f"{cells[k][n]['ettr'] * 100:.1f}%" for k in cells) + " |" for n in names]
    return "\n".join(lines)
