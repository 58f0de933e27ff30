"""Half-open integer intervals and partitions of ``[0, n)``.

Every layout question in the framework -- heterogeneous-TP pipeline boundaries, shard-aligned
gradient reduction between replicas with different TP degrees, optimizer-state resharding,
checkpoint reshard-on-load -- is a question about how two partitions of the same index range
overlap.  Mirrors the interval algebra of the reference (``resihp/utils/intervals.py:17-93``):
``even_split`` puts the remainder on the first parts, exactly like Megatron-style uneven
shards, so both frameworks agree on who owns which row.
"""

from __future__ import annotations

from bisect import bisect_right
from typing import Iterable, Sequence

Interval = tuple[int, int]


def even_split(n: int, k: int) -> list[Interval]:
    """Cut ``[0, n)`` into ``k`` contiguous parts; parts ``0 .. n % k - 1`` get one extra element."""
    if k <= 0:
        raise ValueError(f"number of parts must be positive, got {k}")
    if n < 0:
        raise ValueError(f"length must be non-negative, got {n}")
    q, r = divmod(n, k)
    bounds = [i * q + min(i, r) for i in range(k + 1)]
    return list(zip(bounds[:-1], bounds[1:]))


def length(iv: Interval) -> int:
    return iv[1] - iv[0]


def intersect(a: Interval, b: Interval) -> Interval | None:
    lo = a[0] if a[0] > b[0] else b[0]
    hi = a[1] if a[1] < b[1] else b[1]
    return (lo, hi) if lo < hi else None


def contains(outer: Interval, inner: Interval) -> bool:
    return outer[0] <= inner[0] and inner[1] <= outer[1]


def overlaps(src: Sequence[Interval], dst: Sequence[Interval]) -> list[tuple[int, int, Interval]]:
    """``(i, j, overlap)`` for every non-empty ``src[i] & dst[j]``, ordered by overlap start."""
    found = []
    for i, a in enumerate(src):
        for j, b in enumerate(dst):
            o = intersect(a, b)
            if o is not None:
                found.append((o[0], i, j, o))
    found.sort()
    return [(i, j, o) for _, i, j, o in found]


def refine(partitions: Iterable[Sequence[Interval]]) -> list[Interval]:
    """Coarsest common refinement of partitions that all cover the same range."""
    cuts: set[int] = set()
    span = None
    for part in partitions:
        if not part:
            continue
        s = (part[0][0], part[-1][1])
        if span is None:
            span = s
        elif s != span:
            raise ValueError(f"partitions cover different ranges: {span} vs {s}")
        for lo, hi in part:
            cuts.add(lo)
            cuts.add(hi)
    pts = sorted(cuts)
    return [(a, b) for a, b in zip(pts, pts[1:]) if a < b]


def locate(partition: Sequence[Interval], iv: Interval) -> int:
    """Index of the part that holds all of ``iv``; raises if ``iv`` straddles parts."""
    starts = [p[0] for p in partition]
    k = bisect_right(starts, iv[0]) - 1
    if 0 <= k < len(partition) and contains(partition[k], iv):
        return k
    for idx, part in enumerate(partition):  # partitions need not be sorted
        if contains(part, iv):
            return idx
    raise ValueError(f"{iv} is not inside a single part of {list(partition)}")


def narrow(t, dim: int, iv: Interval, offset: int = 0):
    """View of ``t`` for global interval ``iv`` along ``dim`` when ``t`` starts at ``offset``."""
    return t.narrow(dim, iv[0] - offset, iv[1] - iv[0])


def is_partition(parts: Sequence[Interval], n: int) -> bool:
    if not parts:
        return n == 0
    if parts[0][0] != 0 or parts[-1][1] != n:
        return False
    return all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
