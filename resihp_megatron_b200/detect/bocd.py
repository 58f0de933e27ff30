"""Bayesian online change-point detection (Adams & MacKay, 2007, arXiv:0710.3742).

Model: Gaussian observations with unknown mean and variance under a Normal-Inverse-Gamma prior,
so each run length's posterior predictive is a Student-t; a constant hazard; the run-length
posterior is truncated at ``rmax`` hypotheses so an update costs O(rmax).  Everything is kept in
log space.  The per-run-length sufficient statistics live as columns of one ``[4, R]`` array:
mean ``mu``, pseudo-count ``kappa``, shape ``alpha`` and scale ``beta``.
Parity: ``resihp/detect/bocd.py:30-83`` (same model, prior and truncation).
"""

from __future__ import annotations

import copy
import math

import numpy as np
from scipy.special import gammaln, logsumexp

_MU, _KAPPA, _ALPHA, _BETA = range(4)


def student_t_logpdf(x: float, df: np.ndarray, loc: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """log density of a location-scale Student-t at ``x``."""
    half = 0.5 * (df + 1.0)
    norm = gammaln(half) - gammaln(0.5 * df) - 0.5 * np.log(math.pi * df) - np.log(scale)
    return norm - half * np.log1p(((x - loc) / scale) ** 2 / df)


class BOCD:
    def __init__(self, hazard: float = 1 / 250, mu0: float = 0.0, kappa0: float = 1.0, alpha0: float = 2.0,
                 sigma0: float = 0.03, rmax: int = 400):
        self.log_h, self.log_1mh = math.log(hazard), math.log1p(-hazard)
        # the prior's (mu, kappa, alpha, beta): beta = alpha * sigma^2 puts the prior variance at sigma^2
        self.prior = np.array([mu0, kappa0, alpha0, alpha0 * sigma0 * sigma0])
        self.rmax = rmax
        self.reset()

    def reset(self) -> None:
        self.stats = self.prior[:, None].copy()
        self.log_r = np.zeros(1)
        self.t = 0

    # views kept for callers that read the statistics by name
    @property
    def mu(self) -> np.ndarray:
        return self.stats[_MU]

    def snapshot(self) -> "BOCD":
        return copy.deepcopy(self)

    def _predictive(self, x: float) -> np.ndarray:
        mu, kappa, alpha, beta = self.stats
        scale = np.sqrt(beta * (kappa + 1.0) / (alpha * kappa))
        return student_t_logpdf(x, 2.0 * alpha, mu, scale)

    def _posterior(self, x: float) -> np.ndarray:
        """Statistics after ``x`` for every grown run length, with the prior prepended (r = 0)."""
        mu, kappa, alpha, beta = self.stats
        kappa1 = kappa + 1.0
        grown = np.stack([(kappa * mu + x) / kappa1, kappa1, alpha + 0.5,
                          beta + kappa * (x - mu) ** 2 / (2.0 * kappa1)])
        return np.concatenate([self.prior[:, None], grown], axis=1)

    def update(self, x: float) -> np.ndarray:
        """Add one observation; returns P(r_t = r) for every retained run length r."""
        joint = self.log_r + self._predictive(x)
        log_r = np.concatenate([[logsumexp(joint + self.log_h)], joint + self.log_1mh])
        stats = self._posterior(x)
        if log_r.size > self.rmax:
            log_r, stats = log_r[:self.rmax], stats[:, :self.rmax]
        self.log_r = log_r - logsumexp(log_r)
        self.stats = stats
        self.t += 1
        return np.exp(self.log_r)

    def prob_recent_change(self, window: int) -> float:
        """P(run length <= window): a change point within the last ``window`` observations."""
        return float(np.exp(logsumexp(self.log_r[:window + 1])))

    def map_run_length(self) -> int:
        return int(self.log_r.argmax())

    def segment_mean(self) -> float:
        return float(self.stats[_MU, self.map_run_length()])
