"""Stable tensor identities and plan-derived ownership.

A tensor is named independently of stage boundaries, ``layers.<global layer>.<param>``, and
described by its global shape and TP partition dimension (``None``: replicated).
``holdings(plan)`` lists which device holds which interval of every key -- a replicated tensor
is held as the interval ``(0, 1)``, and every CP slice holds its own copy -- so the old and the
new plan of a reconfiguration determine exactly which state has to move.
Parity: ``resihp/state/layer_registry.py:21-79`` (same keys, specs and holdings).
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass
from typing import Callable

from ..utils.intervals import even_split

FULL = (0, 1)


@dataclass(frozen=True)
class TensorSpec:
    key: str
    global_shape: tuple[int, ...]
    dim: int | None
    trainable: bool = True  # non-trainable tensors (amax history, router bias) carry no optimizer state

    @property
    def extent(self) -> int:
        """Length of the partitioned dimension (1 for a replicated tensor)."""
        return 1 if self.dim is None else self.global_shape[self.dim]

    def local_shape(self, interval: tuple[int, int]) -> tuple[int, ...]:
        if self.dim is None:
            return self.global_shape
        lo, hi = interval
        return self.global_shape[:self.dim] + (hi - lo,) + self.global_shape[self.dim + 1:]

    def split(self, parts: int) -> list[tuple[int, int]]:
        """The interval each of ``parts`` TP ranks holds."""
        return [FULL] * parts if self.dim is None else even_split(self.extent, parts)


Holdings = dict[str, list[tuple[str, tuple[int, int]]]]


def holdings(plan, specs: dict[str, TensorSpec], layer_of: Callable[[str], int]) -> Holdings:
    """key -> sorted ``(device, interval)`` pairs of every holder under ``plan``."""
    keys_of_layer: dict[int, list[str]] = defaultdict(list)
    for key in specs:
        keys_of_layer[layer_of(key)].append(key)
    held: Holdings = defaultdict(list)
    for g in plan.stage_groups:
        lo, hi = g.layers
        for layer in range(lo, hi):
            for key in keys_of_layer.get(layer, ()):
                pieces = specs[key].split(g.tp)
                for c in range(g.cp):
                    held[key].extend(zip(g.slice(c), pieces))
    return {key: sorted(pairs) for key, pairs in held.items()}


def device_layout(h: Holdings, device: str) -> dict[str, tuple[int, int]]:
    """The interval of every key that ``device`` holds."""
    mine = {}
    for key, pairs in h.items():
        for dev, interval in pairs:
            if dev == device:
                mine[key] = interval
    return mine


def reference_specs(cfg) -> dict[str, TensorSpec]:
    """Specs of the CPU reference model (``runtime.reference_model``), plus each layer's fp8 amax
    history when the config keeps one."""
    from ..runtime.reference_model import PARAM_DIMS, full_layer_params

    specs = {}
    for layer in range(cfg.num_layers):
        prefix = f"layers.{layer}."
        for name, tensor in full_layer_params(cfg, layer).items():
            specs[prefix + name] = TensorSpec(prefix + name, tuple(tensor.shape), PARAM_DIMS[name])
        if cfg.amax_history:
            specs[prefix + "amax_history"] = TensorSpec(prefix + "amax_history", (cfg.amax_history,), None,
                                                         trainable=False)
    return specs


def reference_layer_of(key: str) -> int:
    return int(key.split(".", 2)[1])
