"""TP subgroup selection after failures or slowdowns, any degree (no power-of-two rule).

``select_subgroup`` implements Eq. 4 of ResiHP: over the feasible degrees ``k``, take the ``k``
fastest candidates (``k * cp`` with context parallelism) and score the group by its throughput
``k * eff(k) * (slowest member's speed)``.  The best score wins; a near-tie goes to the larger
degree (more memory headroom).  Among equally fast devices the incumbents of the old group rank
first, so a transition moves as little state as possible.  The memory helpers give the smallest
degree a stage fits in and the most layers a group can hold.
Parity: ``resihp/plan/tp_select.py:19-81`` (same selection rule and memory tests).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from .model_spec import ModelProfile, ModelSpec

_TIE = 1e-12


@dataclass(frozen=True)
class TPChoice:
    devices: tuple[str, ...]
    tp: int
    score: float
    standby: tuple[str, ...]


def _is_pow2(k: int) -> bool:
    return k & (k - 1) == 0


def feasible_degrees(model: ModelSpec | None, max_k: int, min_k: int = 1, power_of_two_only: bool = False) -> list[int]:
    """TP degrees in ``[min_k, max_k]`` the model's layout can be split by."""
    ks = range(max(1, min_k), max_k + 1)
    return [k for k in ks if (not power_of_two_only or _is_pow2(k)) and (model is None or model.tp_feasible(k))]


def _per_gpu_bytes(model: ModelSpec, layers: int, tp: int, inflight: int, dp_shard: int, sp: bool,
                   extra: int) -> float:
    return model.static_bytes(layers, tp, dp_shard, extra) + inflight * model.activation_bytes(layers, tp, sp)


def min_tp_for_memory(model: ModelSpec, layers: int, capacity_bytes: float, inflight: int, *, dp_shard: int = 1,
                      sequence_parallel: bool = True, extra_params: int = 0, max_k: int = 64) -> int | None:
    """Smallest feasible TP degree at which ``layers`` layers fit ``capacity_bytes`` per GPU."""
    if math.isinf(capacity_bytes):
        return 1
    fitting = (k for k in feasible_degrees(model, max_k)
               if _per_gpu_bytes(model, layers, k, inflight, dp_shard, sequence_parallel, extra_params)
               <= capacity_bytes)
    return next(fitting, None)


def max_layers_for_memory(model: ModelSpec, tp: int, capacity_bytes: float, inflight: int, *, dp_shard: int = 1,
                          sequence_parallel: bool = True, extra_params: int = 0) -> int:
    """Most layers a TP-``tp`` group can hold (memory grows with the layer count)."""
    if math.isinf(capacity_bytes):
        return model.num_layers
    layers = 0
    while layers < model.num_layers and _per_gpu_bytes(model, layers + 1, tp, inflight, dp_shard,
                                                       sequence_parallel, extra_params) <= capacity_bytes:
        layers += 1
    return layers


def select_subgroup(candidates: list[tuple[str, float]], degrees: list[int], profile: ModelProfile | None = None,
                    incumbents: set[str] | None = None, cp: int = 1) -> TPChoice | None:
    """Best ``TPChoice`` over ``degrees`` for ``(device, speed)`` candidates, or None."""
    keep = incumbents or set()
    order = sorted(candidates, key=lambda dv: (-dv[1], dv[0] not in keep, dv[0]))

    def throughput(k: int, slowest: float) -> float:
        return cp * (profile.group_speed(k, slowest) if profile is not None else k * slowest)

    options = []
    for k in sorted(set(degrees)):
        width = k * cp
        if k < 1 or width > len(order):
            continue
        slowest = order[width - 1][1]  # sorted by speed, descending
        if slowest > 0:
            options.append((k, width, throughput(k, slowest)))
    if not options:
        return None
    top = max(score for _, _, score in options)
    k, width, score = max((o for o in options if o[2] >= top - _TIE), key=lambda o: o[0])
    return TPChoice(tuple(d for d, _ in order[:width]), k, score, tuple(d for d, _ in order[width:]))
