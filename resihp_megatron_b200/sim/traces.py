"""Failure traces scaled from published production statistics.

Fail-stop rates: Llama 3 405B pre-training (Meta, "The Llama 3 Herd of Models", 2024, Table 5):
419 unexpected interruptions in 54 days on 16,384 GPUs, plus 47 planned ones.  Each root-cause
category maps to a failure domain: ``gpu`` (one GPU lost until serviced), ``node`` (all GPUs of
a node), ``network`` (the nodes behind one switch/cable domain) or ``job`` (nothing lost, every
process restarts).  Counts scale linearly with GPUs (per-GPU Poisson processes).  Repair times
and fail-slow statistics are not in the paper: the defaults below are assumptions, exposed as
parameters and swept by the sensitivity study.  (Reference: ``resihp/sim/traces.py:24-146``; the
table is the paper's and therefore identical.)
"""

from __future__ import annotations

import math
import random
from dataclasses import dataclass, field

LLAMA3_GPUS = 16384
LLAMA3_DAYS = 54.0
LLAMA3_PLANNED = 47
# category: (interruptions in the 54-day window, failure domain)
LLAMA3_UNEXPECTED: dict[str, tuple[int, str]] = {
    "faulty_gpu": (148, "gpu"),
    "gpu_hbm3_memory": (72, "gpu"),
    "software_bug": (54, "job"),
    "network_switch_cable": (35, "network"),
    "host_maintenance": (32, "node"),
    "gpu_sram_memory": (19, "gpu"),
    "gpu_system_processor": (17, "gpu"),
    "nic": (7, "node"),
    "nccl_watchdog_timeout": (7, "job"),
    "silent_data_corruption": (6, "gpu"),
    "gpu_thermal_interface_sensor": (6, "gpu"),
    "ssd": (3, "node"),
    "power_supply": (3, "node"),
    "server_chassis": (2, "node"),
    "io_expansion_board": (2, "node"),
    "dependency": (2, "job"),
    "cpu": (2, "node"),
    "system_memory": (2, "node"),
}

_GPU_FAULTS = sum(c for c, d in LLAMA3_UNEXPECTED.values() if d == "gpu")


@dataclass(frozen=True)
class Event:
    t: float
    kind: str                  # fail | slow | planned
    domain: str                # gpu | node | network | job
    category: str
    targets: tuple[int, ...]   # affected GPU indices (empty for job-wide events)
    duration_s: float          # repair time (fail) or slowdown duration (slow)
    factor: float = 1.0        # slowdown factor of a slow event


@dataclass
class TraceConfig:
    gpus: int
    days: float = LLAMA3_DAYS
    gpus_per_node: int = 8
    rate_scale: float = 1.0
    network_domain_nodes: int = 2
    repair_median_s: dict[str, float] = field(default_factory=lambda: {
        "gpu": 24 * 3600.0, "node": 6 * 3600.0, "network": 2 * 3600.0, "job": 0.0})
    repair_sigma: float = 1.0
    # assumption: fail-slow episodes twice as frequent as GPU fail-stops
    slow_per_gpu_day: float = 2.0 * _GPU_FAULTS / (LLAMA3_GPUS * LLAMA3_DAYS)
    slow_factor_median: float = 1.6
    slow_factor_sigma: float = 0.35
    slow_duration_median_s: float = 1800.0
    slow_duration_sigma: float = 1.5
    include_planned: bool = False
    seed: int = 0

    @property
    def nodes(self) -> int:
        return self.gpus // self.gpus_per_node


def per_gpu_day_rates() -> dict[str, float]:
    scale = 1.0 / (LLAMA3_GPUS * LLAMA3_DAYS)
    return {cat: n * scale for cat, (n, _) in LLAMA3_UNEXPECTED.items()}


def expected_failures(gpus: int, days: float) -> float:
    return sum(per_gpu_day_rates().values()) * gpus * days


def _lognormal(rng: random.Random, median: float, sigma: float) -> float:
    return median * math.exp(rng.gauss(0.0, sigma)) if median > 0 else 0.0


def _arrivals(rng: random.Random, rate_per_s: float, horizon: float) -> list[float]:
    out: list[float] = []
    if rate_per_s <= 0:
        return out
    t = rng.expovariate(rate_per_s)
    while t < horizon:
        out.append(t)
        t += rng.expovariate(rate_per_s)
    return out


def _targets(rng: random.Random, domain: str, cfg: TraceConfig) -> tuple[int, ...]:
    gpn = cfg.gpus_per_node
    if domain == "gpu":
        return (rng.randrange(cfg.gpus),)
    if domain == "node":
        n = rng.randrange(cfg.nodes)
        return tuple(range(n * gpn, (n + 1) * gpn))
    if domain == "network":
        k = max(1, min(cfg.network_domain_nodes, cfg.nodes))
        first = rng.randrange(cfg.nodes - k + 1)
        return tuple(range(first * gpn, (first + k) * gpn))
    return ()


def generate(cfg: TraceConfig) -> list[Event]:
    """Deterministic (seeded) event list sorted by time."""
    rng = random.Random(cfg.seed)
    horizon = cfg.days * 86400.0
    events: list[Event] = []
    for cat, rate in per_gpu_day_rates().items():
        domain = LLAMA3_UNEXPECTED[cat][1]
        for t in _arrivals(rng, rate * cfg.rate_scale * cfg.gpus / 86400.0, horizon):
            events.append(Event(t, "fail", domain, cat, _targets(rng, domain, cfg),
                                _lognormal(rng, cfg.repair_median_s[domain], cfg.repair_sigma)))
    for t in _arrivals(rng, cfg.slow_per_gpu_day * cfg.gpus / 86400.0, horizon):
        factor = min(4.0, max(1.1, _lognormal(rng, cfg.slow_factor_median, cfg.slow_factor_sigma)))
        events.append(Event(t, "slow", "gpu", "fail_slow", (rng.randrange(cfg.gpus),),
                            _lognormal(rng, cfg.slow_duration_median_s, cfg.slow_duration_sigma), factor))
    if cfg.include_planned:
        rate = LLAMA3_PLANNED / (LLAMA3_GPUS * LLAMA3_DAYS) * cfg.gpus / 86400.0
        events += [Event(t, "planned", "job", "planned_maintenance", (), 0.0) for t in _arrivals(rng, rate, horizon)]
    events.sort(key=lambda e: e.t)
    return events


def summarize(events: list[Event], cfg: TraceConfig) -> dict:
    fails = [e for e in events if e.kind == "fail"]
    by_domain: dict[str, int] = {}
    for e in fails:
        by_domain[e.domain] = by_domain.get(e.domain, 0) + 1
    hours = cfg.days * 24.0
    return {"gpus": cfg.gpus, "days": cfg.days, "fail_stop": len(fails),
            "fail_slow": sum(1 for e in events if e.kind == "slow"), "by_domain": by_domain,
            "mtbf_h": hours / len(fails) if fails else math.inf,
            "expected_fail_stop": expected_failures(cfg.gpus, cfg.days) * cfg.rate_scale}
