"""Fail-slow detection with workload awareness (all modes share one BOCD core).

* ``greyhound``: change points on the raw (log, warm-up-normalised) iteration time.
* ``paper``: raw series, then drop points within ``validate_ratio`` of the predicted healthy
  time (the published ResiHP filter).
* ``residual``: change points on ``log(T_obs / T_pred)``, removing workload-induced swings
  before detection instead of after it.
After warm-up the noise prior is calibrated from the observed spread; a detection requires
P(change within ``window``) > ``threshold`` and a minimum relative increase measured after the
MAP change point; a cooldown follows each detection.  ``localize`` turns per-group chunk
residuals into normalised throughputs ``p`` for the planner.
(Reference: ``resihp/detect/failslow.py:36-124``.)
"""

from __future__ import annotations

import math
import statistics
from dataclasses import dataclass, field

from .bocd import BOCD
from .predictor import RLSPredictor


@dataclass
class Detection:
    iteration: int
    mode: str
    magnitude: float
    suspects: dict = field(default_factory=dict)


class FailSlowDetector:
    def __init__(self, mode: str = "residual", *, threshold: float = 0.9, window: int = 3, min_increase: float = 0.08,
                 validate_ratio: float = 1.25, warmup: int = 10, sigma0: float = 0.03, hazard: float = 1 / 250,
                 cooldown: int = 10, calibrate: bool = True, sigma_floor: float = 0.005, prior_strength: float = 10.0):
        if mode not in ("greyhound", "paper", "residual"):
            raise ValueError(mode)
        self.mode = mode
        self.threshold = threshold
        self.window = window
        self.min_increase = min_increase
        self.validate_ratio = validate_ratio
        self.warmup = warmup
        self.cooldown = cooldown
        self.hazard = hazard
        self.calibrate = calibrate
        self.sigma_floor = sigma_floor
        self.prior_strength = prior_strength
        self.bocd = BOCD(hazard=hazard, sigma0=sigma0)
        self.xs: list[float] = []
        self._raw_base: list[float] = []
        self.validations = 0
        self.filtered = 0
        self.detections: list[Detection] = []
        self._last = -10 ** 9

    def _value(self, observed: float, predicted: float | None) -> float | None:
        if self.mode == "residual":
            return math.log(observed / predicted) if predicted is not None and predicted > 0 else None
        if len(self._raw_base) < self.warmup:
            self._raw_base.append(observed)
        return math.log(observed / statistics.median(self._raw_base))

    def observe(self, iteration: int, observed: float, predicted: float | None = None) -> Detection | None:
        x = self._value(observed, predicted)
        if x is None:
            return None
        before = self.bocd.snapshot()
        self.bocd.update(x)
        self.xs.append(x)
        if len(self.xs) > 4096:  # long runs: only the recent series is ever compared
            del self.xs[:-2048]
        if self.calibrate and len(self.xs) == self.warmup:
            mean = statistics.fmean(self.xs)
            sigma = max(statistics.pstdev(self.xs), self.sigma_floor)
            self.bocd = BOCD(hazard=self.hazard, mu0=mean, alpha0=self.prior_strength, sigma0=sigma)
            for v in self.xs:
                self.bocd.update(v)
        if len(self.xs) <= self.warmup or iteration - self._last <= self.cooldown:
            return None
        if self.bocd.prob_recent_change(self.window) <= self.threshold:
            return None
        since = min(max(1, self.bocd.map_run_length() + 1), self.window)
        recent = self.xs[-since:]
        base = self.xs[-(since + 4 * self.window):-since] or self.xs[:-since]
        if not base:  # the whole history is one segment: nothing to compare with yet
            return None
        inc = math.exp(statistics.fmean(recent) - statistics.fmean(base)) - 1.0
        if inc < self.min_increase:
            return None
        if self.mode == "paper" and predicted is not None and observed <= self.validate_ratio * predicted:
            self.bocd = before
            self.xs.pop()
            self.filtered += 1
            return None
        self.validations += 1
        self._last = iteration
        det = Detection(iteration, self.mode, 1.0 + inc)
        self.detections.append(det)
        self.bocd.reset()
        return det


def localize(group_samples: dict, predictor: RLSPredictor, speed_factor: dict | None = None,
             threshold: float = 1.1) -> dict:
    """Median observed / expected chunk time per group; groups above ``threshold`` are suspects
    with ``p = expected / observed``."""
    out = {}
    for g, samples in group_samples.items():
        f = (speed_factor or {}).get(g, 1.0)
        ratios = [sec / max(predictor.predict(n, s) / f, 1e-12) for n, s, sec in samples]
        if ratios:
            r = statistics.median(ratios)
            if r > threshold:
                out[g] = 1.0 / r
    return out
