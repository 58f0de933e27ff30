"""Process-group specifications derived from a plan.

Every rank derives the same ordered list of specs from the same plan, so group creation is
deadlock free: creation calls happen in one plan-determined order and ranks outside a group
never block on it.  ``split_layers`` packs groups into layers of pairwise-disjoint rank sets;
each layer is one collective ``split_group`` call (reference: ``resihp/comm/group_spec.py``).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class GroupSpec:
    name: str
    ranks: tuple[int, ...]
    kind: str = "custom"
    keep_singleton: bool = False

    def __post_init__(self) -> None:
        if tuple(sorted(set(self.ranks))) != tuple(self.ranks):
            raise ValueError(f"group {self.name}: ranks must be unique and ascending, got {self.ranks}")

    @property
    def materialized(self) -> bool:
        """Whether a process-group object is created for it (size-1 groups only on request)."""
        return len(self.ranks) > 1 or self.keep_singleton


def canonical_order(specs) -> list[GroupSpec]:
    specs = list(specs)
    if len({s.name for s in specs}) != len(specs):
        raise ValueError("duplicate group names")
    return sorted(specs, key=lambda s: (s.kind, s.name))


def split_layers(specs) -> list[list[GroupSpec]]:
    """First-fit packing of materialised groups into layers of disjoint rank sets; groups with
    an identical rank set are created once."""
    layers: list[tuple[set[int], list[GroupSpec]]] = []
    seen: set[tuple[int, ...]] = set()
    for spec in canonical_order(specs):
        if not spec.materialized or spec.ranks in seen:
            continue
        seen.add(spec.ranks)
        members = set(spec.ranks)
        for taken, layer in layers:
            if not (taken & members):
                layer.append(spec)
                taken |= members
                break
        else:
            layers.append((set(members), [spec]))
    return [layer for _, layer in layers]
