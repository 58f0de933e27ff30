"""Plans precomputed for the failures most likely to come next.

After each commit, ``warm`` plans the survivors of every single-node loss (and, with
``single_device``, of every single-GPU loss) -- on a background thread unless ``blocking``.
A failure that matches a precomputed scenario then gets its plan by one dictionary lookup, which
takes planning off the fail-stop critical path; anything else misses and is planned on the spot.

Entries are tagged with the generation and device set they were computed from; a ``warm`` for a
newer plan invalidates them, and a build still running for an older plan drops its results.
Parity: ``resihp/plan/plan_cache.py:22-86`` (same role and lookup key: the failed-device set).
"""

from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field
from typing import Callable

from .hetero_plan import HeteroParallelPlan
from .topology import ClusterTopology

Replan = Callable[[HeteroParallelPlan, ClusterTopology], HeteroParallelPlan]


@dataclass
class _Epoch:
    """The plan the cached scenarios start from: its generation and the full device set."""

    generation: int
    devices: frozenset
    plans: dict = field(default_factory=dict)  # frozenset(failed ids) -> plan

    def matches(self, generation: int, survivors: set, failed: set) -> bool:
        return generation == self.generation and self.devices - failed == survivors


class PlanCache:
    def __init__(self, replan: Replan, single_device: bool = False):
        self.replan = replan
        self.single_device = single_device
        self.hits = 0
        self.misses = 0
        self.build_seconds = 0.0
        self._mu = threading.Lock()
        self._epoch: _Epoch | None = None
        self._worker: threading.Thread | None = None

    def scenarios(self, plan: HeteroParallelPlan, topology: ClusterTopology) -> list[frozenset[str]]:
        """The failed-device sets to precompute: each node's devices that the plan uses, then
        (optionally) each used device alone."""
        used = set(plan.world)
        per_node = (frozenset(d.id for d in devs) & used for devs in topology.nodes().values())
        todo = [s for s in per_node if s]
        if self.single_device:
            todo.extend(frozenset((d,)) for d in plan.world)
        return todo

    def warm(self, plan: HeteroParallelPlan, topology: ClusterTopology, blocking: bool = False) -> None:
        epoch = _Epoch(plan.generation, frozenset(topology.ids()))
        with self._mu:
            self._epoch = epoch
        if blocking:
            self._fill(epoch, plan, topology)
            return
        self._worker = threading.Thread(target=self._fill, args=(epoch, plan, topology), name="plan-cache",
                                        daemon=True)
        self._worker.start()

    def _current(self, epoch: _Epoch) -> bool:
        with self._mu:
            return self._epoch is epoch

    def _fill(self, epoch: _Epoch, plan: HeteroParallelPlan, topology: ClusterTopology) -> None:
        started = time.monotonic()
        for failed in self.scenarios(plan, topology):
            if not self._current(epoch):
                return  # superseded by a newer plan
            try:
                result = self.replan(plan, topology.without(failed))
            except Exception:  # noqa: BLE001 -- an infeasible scenario is simply not cached
                continue
            with self._mu:
                epoch.plans[failed] = result
        self.build_seconds = time.monotonic() - started

    def wait(self) -> None:
        if self._worker is not None:
            self._worker.join()

    def lookup(self, base_generation: int, topology_ids: set[str], failed: set[str]) -> HeteroParallelPlan | None:
        with self._mu:
            epoch = self._epoch
            found = None
            if epoch is not None and epoch.matches(base_generation, set(topology_ids), set(failed)):
                found = epoch.plans.get(frozenset(failed))
        if found is None:
            self.misses += 1
        else:
            self.hits += 1
        return found
