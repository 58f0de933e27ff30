"""Failure traces scaled from published production statistics.

Fail-stop rates come from Llama 3 405B pre-training (Meta, "The Llama 3 Herd of Models", 2024,
Table 5): 419 unexpected interruptions in 54 days on 16,384 GPUs, plus 47 planned ones.  Each
root-cause category maps to a failure domain -- ``gpu`` (one GPU lost until serviced), ``node``
(every GPU of a node), ``network`` (the nodes behind one switch / cable domain) or ``job``
(nothing lost, every process restarts).  Counts scale linearly with the GPU count (independent
per-GPU Poisson processes).  Repair times and fail-slow statistics are not in the paper; the
defaults below are assumptions, exposed as parameters and swept by the sensitivity study.
Parity: ``resihp/sim/traces.py:24-146`` (the table is the paper's, so the numbers are the same).
"""

from __future__ import annotations

import math
import random
from collections import Counter
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

_GPU_DAYS = LLAMA3_GPUS * LLAMA3_DAYS
_GPU_DOMAIN_FAULTS = sum(n for n, domain in LLAMA3_UNEXPECTED.values() if domain == "gpu")


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
    slow_per_gpu_day: float = 2.0 * _GPU_DOMAIN_FAULTS / _GPU_DAYS
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
    """Interruptions per GPU-day of every category."""
    return {cat: count / _GPU_DAYS for cat, (count, _domain) in LLAMA3_UNEXPECTED.items()}


def expected_failures(gpus: int, days: float) -> float:
    return gpus * days * sum(per_gpu_day_rates().values())


class _Draw:
    """The seeded random choices of one trace."""

    def __init__(self, cfg: TraceConfig):
        self.cfg, self.rng = cfg, random.Random(cfg.seed)

    def lognormal(self, median: float, sigma: float) -> float:
        return median * math.exp(self.rng.gauss(0.0, sigma)) if median > 0 else 0.0

    def poisson_times(self, per_second: float, horizon: float) -> list[float]:
        times, t = [], 0.0
        while per_second > 0:
            t += self.rng.expovariate(per_second)
            if t >= horizon:
                break
            times.append(t)
        return times

    def victims(self, domain: str) -> tuple[int, ...]:
        per_node = self.cfg.gpus_per_node
        if domain == "gpu":
            return (self.rng.randrange(self.cfg.gpus),)
        if domain == "node":
            node = self.rng.randrange(self.cfg.nodes)
            return tuple(range(node * per_node, (node + 1) * per_node))
        if domain == "network":
            width = max(1, min(self.cfg.network_domain_nodes, self.cfg.nodes))
            first = self.rng.randrange(self.cfg.nodes - width + 1)
            return tuple(range(first * per_node, (first + width) * per_node))
        return ()


def generate(cfg: TraceConfig) -> list[Event]:
    """A deterministic (seeded) list of events sorted by time."""
    draw = _Draw(cfg)
    horizon = 86400.0 * cfg.days
    per_second = cfg.gpus / 86400.0
    events: list[Event] = []
    for category, rate in per_gpu_day_rates().items():
        domain = LLAMA3_UNEXPECTED[category][1]
        for t in draw.poisson_times(rate * cfg.rate_scale * per_second, horizon):
            events.append(Event(t, "fail", domain, category, draw.victims(domain),
                                draw.lognormal(cfg.repair_median_s[domain], cfg.repair_sigma)))
    for t in draw.poisson_times(cfg.slow_per_gpu_day * per_second, horizon):
        factor = draw.lognormal(cfg.slow_factor_median, cfg.slow_factor_sigma)
        events.append(Event(t, "slow", "gpu", "fail_slow", (draw.rng.randrange(cfg.gpus),),
                            draw.lognormal(cfg.slow_duration_median_s, cfg.slow_duration_sigma),
                            min(4.0, max(1.1, factor))))
    if cfg.include_planned:
        planned = LLAMA3_PLANNED / _GPU_DAYS * per_second
        events += [Event(t, "planned", "job", "planned_maintenance", (), 0.0)
                   for t in draw.poisson_times(planned, horizon)]
    return sorted(events, key=lambda e: e.t)


def summarize(events: list[Event], cfg: TraceConfig) -> dict:
    fails = [e for e in events if e.kind == "fail"]
    hours = 24.0 * cfg.days
    return {"gpus": cfg.gpus, "days": cfg.days, "fail_stop": len(fails),
            "fail_slow": sum(e.kind == "slow" for e in events), "by_domain": dict(Counter(e.domain for e in fails)),
            "mtbf_h": hours / len(fails) if fails else math.inf,
            "expected_fail_stop": cfg.rate_scale * expected_failures(cfg.gpus, cfg.days)}
