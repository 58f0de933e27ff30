"""Fail-slow detection with workload awareness; all modes share one BOCD core.

Modes differ only in the series the change-point detector watches:

* ``greyhound`` -- the raw iteration time, as ``log(T / median of the warm-up)``;
* ``paper`` -- the same raw series, then a detection is dropped when the observation is within
  ``validate_ratio`` of the predicted healthy time (the published ResiHP filter);
* ``residual`` -- ``log(T_observed / T_predicted)``: the workload-induced swings are removed
  before detection rather than after it.

After ``warmup`` samples the detector's noise prior is calibrated on the observed spread.  A
detection needs P(change within ``window``) > ``threshold`` and a relative increase of at least
``min_increase`` of the samples after the MAP change point over the ones before it; a cooldown
follows each detection.  ``localize`` converts per-group chunk residuals into normalised
throughputs ``p`` for the planner.
Parity: ``resihp/detect/failslow.py:36-124`` (same modes, calibration and acceptance tests).
"""

from __future__ import annotations

import math
import statistics
from dataclasses import dataclass, field

from .bocd import BOCD
from .predictor import RLSPredictor

_MAX_SERIES, _KEEP_SERIES = 4096, 2048


@dataclass
class Detection:
    iteration: int
    mode: str
    magnitude: float
    suspects: dict = field(default_factory=dict)


class _Residual:
    def value(self, observed: float, predicted: float | None) -> float | None:
        if predicted is None or predicted <= 0:
            return None
        return math.log(observed / predicted)


class _Raw:
    def __init__(self, warmup: int):
        self.warmup, self.baseline = warmup, []

    def value(self, observed: float, predicted: float | None) -> float:
        if len(self.baseline) < self.warmup:
            self.baseline.append(observed)
        return math.log(observed / statistics.median(self.baseline))


class FailSlowDetector:
    def __init__(self, mode: str = "residual", *, threshold: float = 0.9, window: int = 3, min_increase: float = 0.08,
                 validate_ratio: float = 1.25, warmup: int = 10, sigma0: float = 0.03, hazard: float = 1 / 250,
                 cooldown: int = 10, calibrate: bool = True, sigma_floor: float = 0.005, prior_strength: float = 10.0):
        if mode not in ("greyhound", "paper", "residual"):
            raise ValueError(mode)
        self.mode = mode
        self.threshold, self.window, self.min_increase = threshold, window, min_increase
        self.validate_ratio, self.warmup, self.cooldown = validate_ratio, warmup, cooldown
        self.hazard, self.calibrate = hazard, calibrate
        self.sigma_floor, self.prior_strength = sigma_floor, prior_strength
        self._series = _Residual() if mode == "residual" else _Raw(warmup)
        self.bocd = BOCD(hazard=hazard, sigma0=sigma0)
        self.xs: list[float] = []
        self.validations = 0
        self.filtered = 0
        self.detections: list[Detection] = []
        self._last = -(10 ** 9)

    def _recalibrate(self) -> None:
        """Replace the prior by one centred on the warm-up samples, with their spread."""
        spread = max(statistics.pstdev(self.xs), self.sigma_floor)
        self.bocd = BOCD(hazard=self.hazard, mu0=statistics.fmean(self.xs), alpha0=self.prior_strength, sigma0=spread)
        for x in self.xs:
            self.bocd.update(x)

    def _increase(self) -> float | None:
        """Relative increase of the samples since the MAP change point (at most ``window`` of
        them) over the ``4 * window`` samples before; None when there is nothing before."""
        since = min(max(1, self.bocd.map_run_length() + 1), self.window)
        after = self.xs[-since:]
        before = self.xs[-(since + 4 * self.window):-since] or self.xs[:-since]
        if not before:
            return None
        return math.expm1(statistics.fmean(after) - statistics.fmean(before))

    def observe(self, iteration: int, observed: float, predicted: float | None = None) -> Detection | None:
        x = self._series.value(observed, predicted)
        if x is None:
            return None
        rollback = self.bocd.snapshot()
        self.bocd.update(x)
        self.xs.append(x)
        if len(self.xs) > _MAX_SERIES:  # long runs: only the recent part is ever compared
            self.xs = self.xs[-_KEEP_SERIES:]
        if self.calibrate and len(self.xs) == self.warmup:
            self._recalibrate()
        if len(self.xs) <= self.warmup or iteration - self._last <= self.cooldown:
            return None
        if self.bocd.prob_recent_change(self.window) <= self.threshold:
            return None
        rise = self._increase()
        if rise is None or rise < self.min_increase:
            return None
        if self.mode == "paper" and predicted is not None and observed <= self.validate_ratio * predicted:
            self.bocd = rollback  # the published filter: forget the point entirely
            self.xs.pop()
            self.filtered += 1
            return None
        self.validations += 1
        self._last = iteration
        found = Detection(iteration, self.mode, 1.0 + rise)
        self.detections.append(found)
        self.bocd.reset()
        return found


def localize(group_samples: dict, predictor: RLSPredictor, speed_factor: dict | None = None,
             threshold: float = 1.1) -> dict:
    """Median observed / expected chunk time per group; the groups above ``threshold`` are the
    suspects, with ``p = expected / observed``."""
    factors = speed_factor or {}
    suspects = {}
    for group, samples in group_samples.items():
        if not samples:
            continue
        scale = factors.get(group, 1.0)
        slowdown = statistics.median(sec / max(predictor.predict(n, s) / scale, 1e-12) for n, s, sec in samples)
        if slowdown > threshold:
            suspects[group] = 1.0 / slowdown
    return suspects
