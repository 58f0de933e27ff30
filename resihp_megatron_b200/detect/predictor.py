"""Online, workload-aware execution-time predictor.

Per micro-batch chunk ``T = alpha * N + beta * sum(l_i^2) + gamma``: ``N`` packed tokens and
``l_i`` the document lengths (attention is block-diagonal under packing).  The coefficients are
fitted by recursive least squares with exponential forgetting (the standard Kalman-gain form,
e.g. Haykin, *Adaptive Filter Theory*, ch. 10) on scaled features.  Updates are gated: once
warmed up, a sample whose log residual exceeds ``gate`` is not learned from -- otherwise the
model would adapt to a fail-slow GPU and hide it.
Parity: ``resihp/detect/predictor.py`` (same model, gate and defaults).
"""

from __future__ import annotations

import math

import numpy as np


class RLSPredictor:
    def __init__(self, scales: tuple[float, ...] = (1e4, 1e8, 1.0), forgetting: float = 0.995, delta: float = 1e4,
                 gate: float = 0.15, warmup: int = 8):
        self.scales = np.asarray(scales, dtype=np.float64)
        self.lam = forgetting
        self.gate, self.warmup = gate, warmup
        dim = self.scales.size
        self.theta = np.zeros(dim)
        self.P = delta * np.eye(dim)  # inverse correlation matrix
        self.n = 0
        self.rejected = 0

    def features(self, tokens: float, sum_sq: float) -> np.ndarray:
        return np.array([tokens, sum_sq, 1.0]) / self.scales

    def predict(self, tokens: float, sum_sq: float) -> float:
        return float(self.features(tokens, sum_sq) @ self.theta)

    def _outlier(self, seconds: float, predicted: float) -> bool:
        if self.n < self.warmup or predicted <= 0:
            return False
        return abs(math.log(max(seconds, 1e-12) / predicted)) > self.gate

    def update(self, tokens: float, sum_sq: float, seconds: float, force: bool = False) -> bool:
        """Learn from one sample; False when the gate rejected it."""
        phi = self.features(tokens, sum_sq)
        predicted = float(phi @ self.theta)
        if not force and self._outlier(seconds, predicted):
            self.rejected += 1
            return False
        p_phi = self.P @ phi
        k = p_phi / (self.lam + float(phi @ p_phi))
        self.theta = self.theta + (seconds - predicted) * k
        self.P = (self.P - np.outer(k, p_phi)) / self.lam
        self.n += 1
        return True

    def coefficients(self) -> tuple[float, float, float]:
        alpha, beta, gamma = (self.theta / self.scales).tolist()
        return alpha, beta, gamma


def fit_least_squares(samples: list[tuple[float, float, float]]) -> tuple[float, float, float]:
    """Batch ``(alpha, beta, gamma)`` from ``(tokens, sum_sq, seconds)`` samples (warm start,
    profiling from device timings)."""
    data = np.asarray(samples, dtype=np.float64)
    design = np.column_stack([data[:, 0], data[:, 1], np.ones(len(data))])
    coef = np.linalg.lstsq(design, data[:, 2], rcond=None)[0]
    return tuple(float(c) for c in coef)
