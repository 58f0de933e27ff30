"""Precomputed plans for the failures most likely to come next.

After each commit a background thread computes the replan for every single-node loss (and,
optionally, every single-device loss); a matching failure then gets its plan in O(1), which
takes planning off the fail-stop critical path.  Anything else is planned synchronously.
(Reference: ``resihp/plan/plan_cache.py:22-86``.)
"""

from __future__ import annotations

import threading
import time
from typing import Callable

from .hetero_plan import HeteroParallelPlan
from .topology import ClusterTopology


class PlanCache:
    def __init__(self, replan: Callable[[HeteroParallelPlan, ClusterTopology], HeteroParallelPlan],
                 single_device: bool = False):
        self.replan = replan
        self.single_device = single_device
        self._lock = threading.Lock()
        self._entries: dict[frozenset[str], HeteroParallelPlan] = {}
        self._base: tuple[int, frozenset[str]] | None = None
        self._thread: threading.Thread | None = None
        self.hits = 0
        self.misses = 0
        self.build_seconds = 0.0

    def scenarios(self, plan: HeteroParallelPlan, topology: ClusterTopology) -> list[frozenset[str]]:
        used = set(plan.world)
        out = [frozenset(d.id for d in devs if d.id in used) for devs in topology.nodes().values()]
        out = [s for s in out if s]
        if self.single_device:
            out += [frozenset([d]) for d in plan.world]
        return out

    def warm(self, plan: HeteroParallelPlan, topology: ClusterTopology, blocking: bool = False) -> None:
        base = (plan.generation, frozenset(topology.ids()))
        with self._lock:
            self._base = base
            self._entries = {}

        def build() -> None:
            t0 = time.monotonic()
            for failed in self.scenarios(plan, topology):
                with self._lock:
                    if self._base != base:
                        return  # a newer plan superseded this one
                try:
                    p = self.replan(plan, topology.without(failed))
                except Exception:  # noqa: BLE001 - infeasible scenarios simply miss
                    continue
                with self._lock:
                    if self._base == base:
                        self._entries[failed] = p
            self.build_seconds = time.monotonic() - t0

        if blocking:
            build()
        else:
            self._thread = threading.Thread(target=build, name="plan-cache", daemon=True)
            self._thread.start()

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()

    def lookup(self, base_generation: int, topology_ids: set[str], failed: set[str]) -> HeteroParallelPlan | None:
        with self._lock:
            base = self._base
            valid = base is not None and base[0] == base_generation and set(base[1]) - set(failed) == set(topology_ids)
            hit = self._entries.get(frozenset(failed)) if valid else None
        if hit is None:
            self.misses += 1
        else:
            self.hits += 1
        return hit
