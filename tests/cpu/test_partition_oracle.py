"""The layer partitioner against exhaustive search on small cases: the returned partition must
attain the lexicographic optimum (bottleneck first, then the sum of squared stage times) of
every contiguous split that respects the per-stage layer bounds."""

import itertools
import random

import pytest

from resihp_megatron_b200.plan.layer_partition import counts_to_ranges, partition_layers


def _compositions(n, k, lo, his):
    if k == 1:
        if lo <= n <= his[0]:
            yield (n,)
        return
    for first in range(lo, min(his[0], n - lo * (k - 1)) + 1):
        for rest in _compositions(n - first, k - 1, lo, his[1:]):
            yield (first, *rest)


def _score(counts, caps, costs, first, last):
    times = []
    for s, (a, b) in enumerate(counts_to_ranges(list(counts))):
        extra = (first if s == 0 else 0.0) + (last if s == len(counts) - 1 else 0.0)
        times.append((sum(costs[a:b]) + extra) / caps[s])
    return max(times), sum(t * t for t in times)


@pytest.mark.parametrize("seed", range(40))
def test_partition_is_the_exhaustive_optimum(seed):
    rng = random.Random(seed)
    L = rng.randint(3, 12)
    S = rng.randint(1, min(4, L))
    caps = [rng.choice([0.25, 0.5, 1.0, 1.0, 2.0]) for _ in range(S)]
    costs = [rng.choice([1.0, 1.0, 1.5, 0.5]) for _ in range(L)] if seed % 2 else None
    first, last = rng.choice([0.0, 0.5]), rng.choice([0.0, 1.0, 2.0])
    lo = rng.choice([1, 1, 2]) if L >= 2 * S else 1
    his = [rng.randint(lo, L) for _ in range(S)] if seed % 3 == 0 else [L] * S
    options = list(_compositions(L, S, lo, his))
    if not options:
        with pytest.raises(ValueError):
            partition_layers(L, caps, layer_cost=costs, first_extra=first, last_extra=last, max_layers=his,
                             min_layers=lo)
        return
    c = costs or [1.0] * L
    best = min(_score(o, caps, c, first, last) for o in options)
    got = partition_layers(L, caps, layer_cost=costs, first_extra=first, last_extra=last, max_layers=his,
                           min_layers=lo)
    assert sum(got) == L and all(lo <= g <= h for g, h in zip(got, his))
    mx, sq = _score(got, caps, c, first, last)
    assert mx == pytest.approx(best[0], rel=1e-12)
    assert sq == pytest.approx(best[1], rel=1e-9)


def test_ties_prefer_earlier_stages_taking_more_layers():
    # [3, 5, 4] and [3, 4, 5] have the same bottleneck and sum of squares
    assert partition_layers(12, [1.0, 1.0, 1.0], max_layers=[3, 6, 6]) == [3, 5, 4]
