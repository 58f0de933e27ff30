"""Cluster topology: devices grouped into nodes (one NVLink / NVSwitch domain each) and racks
(shared failure domains).

Device ids follow ``n{node}g{gpu}``.  A topology is immutable; ``without`` and ``with_speeds``
return new ones.  Lookups go through an id index built once per instance.
Parity: ``resihp/plan/topology.py:18-53`` (same device record and queries).
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass, field
from typing import Iterable


@dataclass(frozen=True)
class Device:
    """One GPU: its id, the node (NVLink domain) and rack it sits in, its index on the node and
    its relative speed (1.0 = nominal; a fail-slow GPU reports less)."""

    id: str
    node: str
    local_rank: int
    rack: str = "r0"
    speed: float = 1.0


@dataclass(frozen=True)
class ClusterTopology:
    devices: tuple[Device, ...]
    _index: dict = field(init=False, repr=False, compare=False, hash=False)

    def __post_init__(self):
        object.__setattr__(self, "devices", tuple(self.devices))
        object.__setattr__(self, "_index", {d.id: d for d in self.devices})

    # ------------------------------------------------------------------ construction
    @classmethod
    def uniform(cls, num_nodes: int, gpus_per_node: int, nodes_per_rack: int | None = None) -> "ClusterTopology":
        """``num_nodes`` identical nodes of ``gpus_per_node`` GPUs; with ``nodes_per_rack`` the
        nodes fill racks ``r0, r1, ...`` in order, otherwise all share rack ``r0``."""

        def rack(n: int) -> str:
            return f"r{n // nodes_per_rack}" if nodes_per_rack else "r0"

        return cls(tuple(Device(f"n{n}g{g}", f"n{n}", g, rack(n))
                         for n, g in itertools.product(range(num_nodes), range(gpus_per_node))))

    def without(self, failed: Iterable[str]) -> "ClusterTopology":
        drop = frozenset(failed)
        return ClusterTopology(tuple(filter(lambda d: d.id not in drop, self.devices)))

    def with_speeds(self, speeds: dict[str, float]) -> "ClusterTopology":
        def rescored(d: Device) -> Device:
            return d if d.id not in speeds else Device(d.id, d.node, d.local_rank, d.rack, speeds[d.id])

        return ClusterTopology(tuple(map(rescored, self.devices)))

    # ------------------------------------------------------------------ queries
    def ids(self) -> list[str]:
        return list(self._index)

    def by_id(self) -> dict[str, Device]:
        return dict(self._index)

    def node_of(self, dev_id: str) -> str:
        return self._index[dev_id].node

    def speed(self, dev_id: str) -> float:
        return self._index[dev_id].speed

    def nodes(self) -> dict[str, list[Device]]:
        """Node name -> its devices ordered by local rank; nodes in name order."""
        ordered = sorted(self.devices, key=lambda d: (d.node, d.local_rank))
        return {node: list(group) for node, group in itertools.groupby(ordered, key=lambda d: d.node)}
