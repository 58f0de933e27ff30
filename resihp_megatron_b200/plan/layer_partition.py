"""Contiguous layer partition across pipeline stages (ResiHP section 6.2).

Objective, lexicographic: (1) minimise the slowest stage's time, (2) among partitions with that
bottleneck, minimise the sum of squared stage times (the most even spread of the rest).  A
stage's time is ``(sum of its layer costs + extra work) / capacity``, where capacity is the
stage's aggregate speed over its replicas and the extra work is the embedding / LM head charged
to the first / last stage.  Per-stage memory caps bound its layer count from above and
``min_layers`` from below.  Residual imbalance between replicas is removed later by
micro-batch migration.

Algorithm (exact):

1. The optimal bottleneck is one of the finitely many values ``time(s, i, j)``.  Sort them and
   binary-search for the smallest ``T`` for which a partition with every stage ``<= T`` exists;
   feasibility is a reachability sweep over layer prefixes.
2. With ``T`` fixed the second objective is additive, so a suffix dynamic program over
   ``(stage, first layer)`` minimises the sum of squares among stages ``<= T``.  Ties go to the
   partition whose earlier stages take more layers (the last stage also carries the LM head).

Parity: ``resihp/plan/layer_partition.py:14-56`` (same objective and constraints; the reference
uses a single prefix DP over (max, sum of squares) pairs).
"""

from __future__ import annotations

import bisect
import itertools
import math


class _Stages:
    """Stage-time oracle over prefix sums of the layer costs."""

    def __init__(self, num_layers, capacities, layer_cost, first_extra, last_extra, max_layers, min_layers):
        self.L = num_layers
        self.S = len(capacities)
        costs = [1.0] * num_layers if layer_cost is None else list(layer_cost)
        self.prefix = [0.0, *itertools.accumulate(costs)]
        self.cap = [max(float(c), 1e-12) for c in capacities]
        self.extra = [0.0] * self.S
        self.extra[0] += first_extra
        self.extra[-1] += last_extra
        self.hi = list(max_layers) if max_layers is not None else [num_layers] * self.S
        self.lo = min_layers

    def time(self, s: int, i: int, j: int) -> float:
        return (self.prefix[j] - self.prefix[i] + self.extra[s]) / self.cap[s]

    def spans(self, s: int, i: int):
        """Layer counts stage ``s`` may take when it starts at layer ``i``."""
        return range(self.lo, min(self.hi[s], self.L - i) + 1)

    def feasible(self, bound: float) -> bool:
        reach = {0}
        for s in range(self.S):
            reach = {i + c for i in reach for c in self.spans(s, i) if self.time(s, i, i + c) <= bound}
            if not reach:
                return False
        return self.L in reach


def partition_layers(num_layers: int, capacities: list[float], *, layer_cost: list[float] | None = None,
                     first_extra: float = 0.0, last_extra: float = 0.0, max_layers: list[int] | None = None,
                     min_layers: int = 1) -> list[int]:
    """Layer counts per stage (see the module docstring for the objective)."""
    S = len(capacities)
    if S == 0 or num_layers < S * min_layers:
        raise ValueError(f"cannot place {num_layers} layers on {S} stages with at least {min_layers} each")
    st = _Stages(num_layers, capacities, layer_cost, first_extra, last_extra, max_layers, min_layers)
    candidates = sorted({st.time(s, i, i + c) for s in range(S) for i in range(num_layers + 1)
                         for c in st.spans(s, i)})
    if not candidates or not st.feasible(candidates[-1]):
        raise ValueError("no feasible partition under the memory caps")
    lo, hi = 0, len(candidates) - 1  # smallest feasible bottleneck by bisection
    while lo < hi:
        mid = (lo + hi) // 2
        if st.feasible(candidates[mid]):
            hi = mid
        else:
            lo = mid + 1
    bound = candidates[lo]

    # best[s][i]: least sum of squares placing layers [i, L) on stages [s, S) with every stage <= bound
    best = [[math.inf] * (num_layers + 1) for _ in range(S + 1)]
    best[S][num_layers] = 0.0
    for s in range(S - 1, -1, -1):
        for i in range(num_layers + 1):
            for c in st.spans(s, i):
                t = st.time(s, i, i + c)
                if t <= bound and best[s + 1][i + c] < math.inf:
                    best[s][i] = min(best[s][i], t * t + best[s + 1][i + c])
    counts, i = [], 0
    for s in range(S):
        target = best[s][i]
        tol = 1e-12 * max(1.0, abs(target))
        take = max(c for c in st.spans(s, i)
                   if st.time(s, i, i + c) <= bound and
                   st.time(s, i, i + c) ** 2 + best[s + 1][i + c] <= target + tol)
        counts.append(take)
        i += take
    return counts


def counts_to_ranges(counts: list[int]) -> list[tuple[int, int]]:
    """``[2, 3] -> [(0, 2), (2, 5)]``: half-open layer ranges of consecutive stages."""
    ends = list(itertools.accumulate(counts))
    return list(zip([0, *ends[:-1]], ends))
