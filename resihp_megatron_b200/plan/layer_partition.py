"""Layer repartition across pipeline stages.

Exact min-max contiguous partition by dynamic programming over (stage, layer prefix) with
per-stage capacities (aggregated over a stage's replicas), optional per-layer costs, extra
first/last-stage work, per-stage memory caps and a minimum layer count; ties on the maximum
stage time are broken by the smaller sum of squared stage times.  Residual imbalance across
replicas is removed afterwards by micro-batch migration.
(Reference: ``resihp/plan/layer_partition.py:14-56``, ResiHP section 6.2.)
"""

from __future__ import annotations

import math


def partition_layers(num_layers: int, capacities: list[float], *, layer_cost: list[float] | None = None,
                     first_extra: float = 0.0, last_extra: float = 0.0, max_layers: list[int] | None = None,
                     min_layers: int = 1) -> list[int]:
    S = len(capacities)
    if S == 0 or num_layers < S * min_layers:
        raise ValueError(f"cannot place {num_layers} layers on {S} stages with at least {min_layers} each")
    costs = layer_cost if layer_cost is not None else [1.0] * num_layers
    pre = [0.0]
    for c in costs:
        pre.append(pre[-1] + c)
    caps = [max(c, 1e-12) for c in capacities]
    cap_layers = max_layers if max_layers is not None else [num_layers] * S

    def stage_time(s: int, i: int, j: int) -> float:
        extra = (first_extra if s == 0 else 0.0) + (last_extra if s == S - 1 else 0.0)
        return (pre[j] - pre[i] + extra) / caps[s]

    inf = (math.inf, math.inf)
    # f[s][j]: best (max stage time, sum of squares) placing layers [0, j) on stages [0, s)
    f = [[inf] * (num_layers + 1) for _ in range(S + 1)]
    arg = [[-1] * (num_layers + 1) for _ in range(S + 1)]
    f[0][0] = (0.0, 0.0)
    for s in range(S):
        for j in range(num_layers + 1):
            lo = max(0, j - cap_layers[s])
            for i in range(j - min_layers, lo - 1, -1):
                prev = f[s][i]
                if prev[0] == math.inf:
                    continue
                t = stage_time(s, i, j)
                cand = (max(prev[0], t), prev[1] + t * t)
                if cand < f[s + 1][j]:
                    f[s + 1][j] = cand
                    arg[s + 1][j] = i
    if f[S][num_layers][0] == math.inf:
        raise ValueError("no feasible partition under the memory caps")
    counts = []
    j = num_layers
    for s in range(S, 0, -1):
        i = arg[s][j]
        counts.append(j - i)
        j = i
    return counts[::-1]


def counts_to_ranges(counts: list[int]) -> list[tuple[int, int]]:
    out, a = [], 0
    for c in counts:
        out.append((a, a + c))
        a += c
    return out
