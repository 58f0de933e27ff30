"""Initial placement of the (replica, stage) TP groups onto nodes.

Two strategies:

* ``spread`` -- nodes are visited round robin across racks, and groups are handed out stage by
  stage, so the replicas of one stage land on different nodes (different racks when there are
  several).  Losing one node then never removes every copy of a stage, and recovery can take
  the no-rollback path.
* ``megatron`` -- conventional packing (TP fastest, then DP, then PP): consecutive TP slots in
  node order, which puts a stage's replicas next to each other.

``stage_loss_exposure`` is the fraction of single-node losses that take out every replica of
some stage (0.0 for ``spread`` whenever the cluster allows it).
Parity: ``resihp/plan/placement.py:25-60`` (the same two strategies and exposure measure).
"""

from __future__ import annotations

import itertools
from collections import deque

from .topology import ClusterTopology

Key = tuple[int, int]


def _free_slots(topology: ClusterTopology, tp: int) -> dict[str, deque]:
    """Per node, the disjoint runs of ``tp`` consecutive local GPUs still available."""
    out = {}
    for node, devs in topology.nodes().items():
        ids = [d.id for d in devs]
        whole = len(ids) // tp
        out[node] = deque(tuple(ids[k * tp:(k + 1) * tp]) for k in range(whole))
    return out


def _rack_interleaved_nodes(topology: ClusterTopology, nodes) -> list[str]:
    """Nodes ordered r0's first, r1's first, ..., r0's second, ... (racks by name)."""
    rack_of = {d.node: d.rack for d in topology.devices}
    by_rack: dict[str, list[str]] = {}
    for node in sorted(nodes):
        by_rack.setdefault(rack_of[node], []).append(node)
    columns = itertools.zip_longest(*(by_rack[r] for r in sorted(by_rack)))
    return [n for column in columns for n in column if n is not None]


def place_groups(topology: ClusterTopology, num_replicas: int, num_stages: int, tp: int,
                 strategy: str = "spread") -> dict[Key, tuple[str, ...]]:
    """Map every ``(replica, stage)`` to the device ids of its TP group."""
    if strategy not in ("spread", "megatron"):
        raise ValueError(f"unknown placement strategy {strategy!r}")
    free = _free_slots(topology, tp)
    wanted = [(r, s) for s in range(num_stages) for r in range(num_replicas)]
    available = sum(map(len, free.values()))
    if available < len(wanted):
        raise ValueError(f"need {len(wanted)} TP{tp} slots, the cluster has {available}")
    if strategy == "megatron":
        packed = itertools.chain.from_iterable(free[n] for n in sorted(free))
        return dict(zip(wanted, packed))
    ring = deque(n for n in _rack_interleaved_nodes(topology, free) if free[n])
    placement: dict[Key, tuple[str, ...]] = {}
    for key in wanted:
        node = ring.popleft()
        placement[key] = free[node].popleft()
        if free[node]:
            ring.append(node)  # back of the ring: the next group goes to the next node
    return placement


def stage_loss_exposure(placement: dict[Key, tuple[str, ...]], topology: ClusterTopology) -> float:
    """Fraction of single-node failures that remove every replica of at least one stage."""
    node_of = {d.id: d.node for d in topology.devices}
    nodes_of_group = {key: {node_of[d] for d in devs} for key, devs in placement.items()}
    stages: dict[int, list[set]] = {}
    for (_, stage), nodes in nodes_of_group.items():
        stages.setdefault(stage, []).append(nodes)
    all_nodes = set().union(*nodes_of_group.values()) if nodes_of_group else set()
    if not all_nodes:
        return 0.0

    def fatal(node: str) -> bool:
        return any(all(node in g for g in groups) for groups in stages.values())

    return sum(map(fatal, all_nodes)) / len(all_nodes)
