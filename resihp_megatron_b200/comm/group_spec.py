"""Process-group specifications derived from a plan.

Every rank derives the same ordered list of specs from the same plan, which makes group
creation deadlock free: the creation calls happen in one plan-determined order, and ranks
outside a group never block on it.  ``split_layers`` packs the groups into layers of pairwise
disjoint rank sets (first fit in canonical order); each layer is created by one collective
``split_group`` call.
Parity: ``resihp/comm/group_spec.py`` (same spec fields and canonical order).
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass
from itertools import count


@dataclass(frozen=True)
class GroupSpec:
    name: str
    ranks: tuple[int, ...]
    kind: str = "custom"
    keep_singleton: bool = False

    def __post_init__(self) -> None:
        ascending = all(a < b for a, b in zip(self.ranks, self.ranks[1:]))
        if not ascending:
            raise ValueError(f"group {self.name}: ranks must be unique and ascending, got {self.ranks}")

    @property
    def materialized(self) -> bool:
        """Whether a process-group object is created (a size-1 group only on request)."""
        return self.keep_singleton or len(self.ranks) > 1


def canonical_order(specs) -> list[GroupSpec]:
    specs = list(specs)
    names = [s.name for s in specs]
    if len(set(names)) < len(names):
        raise ValueError("duplicate group names")
    return sorted(specs, key=lambda s: (s.kind, s.name))


def split_layers(specs) -> list[list[GroupSpec]]:
    """Materialised groups packed into layers of disjoint rank sets: each group goes to the
    first layer none of its ranks is in yet; a rank set seen before is not created again."""
    layers: list[list[GroupSpec]] = []
    layers_of_rank: dict[int, set[int]] = defaultdict(set)
    created: set[tuple[int, ...]] = set()
    for spec in canonical_order(specs):
        if not spec.materialized or spec.ranks in created:
            continue
        created.add(spec.ranks)
        busy = set().union(*(layers_of_rank[r] for r in spec.ranks))
        k = next(i for i in count() if i not in busy)
        if k == len(layers):
            layers.append([])
        layers[k].append(spec)
        for r in spec.ranks:
            layers_of_rank[r].add(k)
    return layers
