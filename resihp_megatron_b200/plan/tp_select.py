"""TP subgroup selection after failures / slowdowns, without the power-of-two restriction.

``select_subgroup`` maximises ``k * eff(k) * min_{i in S_k} p_i`` over TP degrees ``k`` where
``S_k`` is the top-``k`` devices by normalised speed (Eq. 4 of ResiHP); ties go to the larger
group (more memory headroom), and among equally fast devices incumbents are kept so the
transition moves the least state.  With context parallelism a degree ``k`` takes ``k * cp``
devices.  Memory helpers give the smallest TP degree that fits and the most layers a group can
hold.  (Reference: ``resihp/plan/tp_select.py:19-81``.)
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from .model_spec import ModelProfile, ModelSpec


@dataclass(frozen=True)
class TPChoice:
    devices: tuple[str, ...]
    tp: int
    score: float
    standby: tuple[str, ...]


def feasible_degrees(model: ModelSpec | None, max_k: int, min_k: int = 1, power_of_two_only: bool = False) -> list[int]:
    out = []
    for k in range(max(1, min_k), max_k + 1):
        if power_of_two_only and (k & (k - 1)):
            continue
        if model is None or model.tp_feasible(k):
            out.append(k)
    return out


def _fits(model: ModelSpec, layers: int, tp: int, capacity: float, inflight: int, dp_shard: int, sp: bool,
          extra: int) -> bool:
    need = model.static_bytes(layers, tp, dp_shard, extra) + inflight * model.activation_bytes(layers, tp, sp)
    return need <= capacity


def min_tp_for_memory(model: ModelSpec, layers: int, capacity_bytes: float, inflight: int, *, dp_shard: int = 1,
                      sequence_parallel: bool = True, extra_params: int = 0, max_k: int = 64) -> int | None:
    if math.isinf(capacity_bytes):
        return 1
    for k in range(1, max_k + 1):
        if model.tp_feasible(k) and _fits(model, layers, k, capacity_bytes, inflight, dp_shard, sequence_parallel,
                                          extra_params):
            return k
    return None


def max_layers_for_memory(model: ModelSpec, tp: int, capacity_bytes: float, inflight: int, *, dp_shard: int = 1,
                          sequence_parallel: bool = True, extra_params: int = 0) -> int:
    if math.isinf(capacity_bytes):
        return model.num_layers
    best = 0
    for layers in range(1, model.num_layers + 1):
        if not _fits(model, layers, tp, capacity_bytes, inflight, dp_shard, sequence_parallel, extra_params):
            break
        best = layers
    return best


def select_subgroup(candidates: list[tuple[str, float]], degrees: list[int], profile: ModelProfile | None = None,
                    incumbents: set[str] | None = None, cp: int = 1) -> TPChoice | None:
    inc = incumbents or set()
    ranked = sorted(candidates, key=lambda c: (-c[1], c[0] not in inc, c[0]))
    best: TPChoice | None = None
    for k in sorted(degrees):
        n = k * cp
        if k < 1 or n > len(ranked):
            continue
        chosen = ranked[:n]
        slowest = min(p for _, p in chosen)
        if slowest <= 0:
            continue
        score = (profile.group_speed(k, slowest) if profile is not None else k * slowest) * cp
        if best is None or score >= best.score - 1e-12:
            best = TPChoice(tuple(d for d, _ in chosen), k, score, tuple(d for d, _ in ranked[n:]))
    return best
