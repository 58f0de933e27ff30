"""Bayesian online change-point detection (Adams & MacKay, 2007, arXiv:0710.3742).

Gaussian observations with unknown mean and variance: Normal-Inverse-Gamma conjugate prior,
Student-t posterior predictive, constant hazard, run-length posterior truncated at ``rmax`` so
each update is O(rmax); all probabilities kept in log space.  (Reference:
``resihp/detect/bocd.py:30-83``.)
"""

from __future__ import annotations

import copy
import math

import numpy as np

_lgamma = np.vectorize(math.lgamma)


def _logsumexp(a: np.ndarray) -> float:
    m = float(np.max(a))
    if not math.isfinite(m):
        return m
    return m + math.log(float(np.sum(np.exp(a - m))))


def student_t_logpdf(x: float, df: np.ndarray, loc: np.ndarray, scale: np.ndarray) -> np.ndarray:
    z2 = ((x - loc) / scale) ** 2
    return (_lgamma((df + 1) / 2) - _lgamma(df / 2) - 0.5 * np.log(df * math.pi) - np.log(scale)
            - (df + 1) / 2 * np.log1p(z2 / df))


class BOCD:
    def __init__(self, hazard: float = 1 / 250, mu0: float = 0.0, kappa0: float = 1.0, alpha0: float = 2.0,
                 sigma0: float = 0.03, rmax: int = 400):
        self.log_h = math.log(hazard)
        self.log_1mh = math.log1p(-hazard)
        self.prior = (mu0, kappa0, alpha0, alpha0 * sigma0 ** 2)  # (mu, kappa, alpha, beta)
        self.rmax = rmax
        self.reset()

    def reset(self) -> None:
        mu0, k0, a0, b0 = self.prior
        self.log_r = np.zeros(1)
        self.mu, self.kappa = np.array([mu0]), np.array([k0])
        self.alpha, self.beta = np.array([a0]), np.array([b0])
        self.t = 0

    def snapshot(self) -> "BOCD":
        return copy.deepcopy(self)

    def update(self, x: float) -> np.ndarray:
        """Add one observation; returns P(r_t = r) for every retained run length r."""
        scale = np.sqrt(self.beta * (self.kappa + 1) / (self.alpha * self.kappa))
        lp = student_t_logpdf(x, 2 * self.alpha, self.mu, scale)
        grow = self.log_r + lp + self.log_1mh
        change = _logsumexp(self.log_r + lp + self.log_h)
        log_r = np.concatenate([[change], grow])
        log_r -= _logsumexp(log_r)
        mu0, k0, a0, b0 = self.prior
        k1 = self.kappa + 1
        self.beta = np.concatenate([[b0], self.beta + self.kappa * (x - self.mu) ** 2 / (2 * k1)])
        self.mu = np.concatenate([[mu0], (self.kappa * self.mu + x) / k1])
        self.kappa = np.concatenate([[k0], k1])
        self.alpha = np.concatenate([[a0], self.alpha + 0.5])
        if len(log_r) > self.rmax:
            log_r = log_r[: self.rmax]
            log_r -= _logsumexp(log_r)
            self.mu, self.kappa, self.alpha, self.beta = (v[: self.rmax] for v in
                                                          (self.mu, self.kappa, self.alpha, self.beta))
        self.log_r = log_r
        self.t += 1
        return np.exp(log_r)

    def prob_recent_change(self, window: int) -> float:
        """P(run length <= window): a change point within the last ``window`` observations."""
        return float(np.exp(_logsumexp(self.log_r[: window + 1])))

    def map_run_length(self) -> int:
        return int(np.argmax(self.log_r))

    def segment_mean(self) -> float:
        return float(self.mu[self.map_run_length()])
