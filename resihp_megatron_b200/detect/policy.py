"""When to act on a confirmed fail-slow: ski rental with hysteresis.

"Renting" keeps paying the per-iteration excess time of the degraded layout; "buying" pays the
reconfiguration once.  Buying as soon as the accumulated excess reaches the reconfiguration
cost is 2-competitive against an oracle that knows how long the slowdown lasts (the classic
ski-rental bound).  ``min_gain`` (a relative improvement below which nothing accumulates) and
``min_dwell`` (iterations between actions) keep noisy or transient slowdowns from causing
oscillation.  Parity: ``resihp/detect/policy.py:22-42`` (same rule and defaults).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class Decision:
    act: bool
    reason: str
    accumulated: float = 0.0


class SkiRentalPolicy:
    def __init__(self, min_gain: float = 0.03, min_dwell: int = 50):
        self.min_gain, self.min_dwell = min_gain, min_dwell
        self.accumulated = 0.0
        self.last_action = -(10 ** 9)

    def observe(self, iteration: int, current_iter_s: float, best_iter_s: float, reconfig_cost_s: float) -> Decision:
        excess = current_iter_s - best_iter_s
        relative = excess / max(current_iter_s, 1e-12)
        if relative < self.min_gain:  # not worth renting toward: start over
            self.accumulated = 0.0
            return Decision(False, f"gain {relative:.3f} below {self.min_gain}")
        self.accumulated += excess
        if iteration - self.last_action < self.min_dwell:
            return Decision(False, "dwell time not elapsed", self.accumulated)
        if self.accumulated < reconfig_cost_s:
            return Decision(False, "renting", self.accumulated)
        paid = self.accumulated
        self.accumulated, self.last_action = 0.0, iteration
        return Decision(True, f"excess {paid:.2f}s >= reconfiguration cost {reconfig_cost_s:.2f}s", paid)
