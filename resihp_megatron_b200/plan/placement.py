"""Initial placement of (replica, stage) TP groups onto nodes.

``spread`` walks nodes interleaved across racks and assigns groups stage-major, so the DP
replicas of a stage land on different nodes (and racks when possible): one node failure then
never removes every live copy of a stage, which keeps recovery on the zero-rollback path.
``megatron`` is the conventional packing (TP fastest, then DP, then PP), which puts the
replicas of a stage on one node.  ``stage_loss_exposure`` measures the difference.
(Reference: ``resihp/plan/placement.py:25-60``.)
"""

from __future__ import annotations

from .topology import ClusterTopology

Key = tuple[int, int]


def _tp_slots(topology: ClusterTopology, tp: int) -> dict[str, list[tuple[str, ...]]]:
    slots = {}
    for node, devs in topology.nodes().items():
        ids = [d.id for d in devs]
        slots[node] = [tuple(ids[i:i + tp]) for i in range(0, len(ids) - tp + 1, tp)]
    return slots


def place_groups(topology: ClusterTopology, num_replicas: int, num_stages: int, tp: int,
                 strategy: str = "spread") -> dict[Key, tuple[str, ...]]:
    slots = _tp_slots(topology, tp)
    need = num_replicas * num_stages
    have = sum(len(v) for v in slots.values())
    if have < need:
        raise ValueError(f"need {need} TP{tp} slots, the cluster has {have}")
    keys = [(r, s) for s in range(num_stages) for r in range(num_replicas)]
    if strategy == "megatron":
        flat = [slot for node in sorted(slots) for slot in slots[node]]
        return dict(zip(keys, flat))
    if strategy != "spread":
        raise ValueError(f"unknown placement strategy {strategy!r}")
    rack_of = {d.node: d.rack for d in topology.devices}
    racks: dict[str, list[str]] = {}
    for node in sorted(slots):
        racks.setdefault(rack_of[node], []).append(node)
    walk = []
    for i in range(max(len(v) for v in racks.values())):
        for rack in sorted(racks):
            if i < len(racks[rack]):
                walk.append(racks[rack][i])
    used = dict.fromkeys(walk, 0)
    out: dict[Key, tuple[str, ...]] = {}
    pos = 0
    for key in keys:
        for _ in range(len(walk)):
            node = walk[pos % len(walk)]
            pos += 1
            if used[node] < len(slots[node]):
                out[key] = slots[node][used[node]]
                used[node] += 1
                break
    return out


def stage_loss_exposure(placement: dict[Key, tuple[str, ...]], topology: ClusterTopology) -> float:
    """Fraction of single-node failures that remove every replica of at least one stage."""
    node_of = {d.id: d.node for d in topology.devices}
    nodes = sorted({node_of[d] for devs in placement.values() for d in devs})
    stages = sorted({s for _, s in placement})
    exposed = 0
    for n in nodes:
        for s in stages:
            replicas = [devs for (r, st), devs in placement.items() if st == s]
            if all(any(node_of[d] == n for d in devs) for devs in replicas):
                exposed += 1
                break
    return exposed / len(nodes) if nodes else 0.0
