"""Iteration-level transactions; the optimizer step is the commit point.

Phases: ``COMPUTE -> REDUCED`` (gradients all-reduced) ``-> STEPPING -> COMMITTED``, or
``ABORTED``.  Reduced gradients are kept until the step commits, which allows roll-forward
recovery without a per-step consensus round: survivors report ``(committed_iteration,
has_reduced_grads)``, and the planner moves everyone to the newest committed iteration -- ranks
that hold that iteration's reduced gradients step locally (Adam is deterministic), the others
copy state from a rank that committed it.

``buffers`` are the non-trainable tensors an iteration mutates (fp8 amax history, MoE router
bias and loads).  They are copied at ``begin`` and put back on rollback -- except after REDUCED,
where the iteration may still roll forward.
Parity: ``resihp/state/transaction.py:22-142`` (same phases, recovery report and roll-forward).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Callable

import torch

from .rng_data import DataCursor, capture_rng_state, restore_rng_state


class TxnPhase(str, Enum):
    COMPUTE = "compute"
    REDUCED = "reduced"
    STEPPING = "stepping"
    COMMITTED = "committed"
    ABORTED = "aborted"


_NEXT = {TxnPhase.COMPUTE: TxnPhase.REDUCED, TxnPhase.REDUCED: TxnPhase.STEPPING,
         TxnPhase.STEPPING: TxnPhase.COMMITTED}


@dataclass
class IterationTransaction:
    iteration: int
    rng: dict
    cursor: dict
    phase: TxnPhase = TxnPhase.COMPUTE
    events: list[str] = field(default_factory=list)
    buffers: dict[str, torch.Tensor] = field(default_factory=dict)


class TransactionManager:
    def __init__(self, cursor: DataCursor | None = None, committed_iteration: int = -1,
                 buffers: Callable[[], dict[str, torch.Tensor]] | None = None):
        self.cursor = cursor if cursor is not None else DataCursor(committed_iteration + 1)
        self.committed_iteration = committed_iteration
        self.current: IterationTransaction | None = None
        self.aborts = 0
        self.buffers = buffers

    def track_buffers(self, buffers: Callable[[], dict[str, torch.Tensor]] | None) -> None:
        self.buffers = buffers

    def _live_buffers(self) -> dict[str, torch.Tensor]:
        return {} if self.buffers is None else self.buffers()

    def _put_back_buffers(self) -> None:
        saved = self.current.buffers if self.current is not None else None
        if not saved:
            return
        with torch.no_grad():
            for key, live in self._live_buffers().items():
                if key in saved:
                    live.copy_(saved[key])

    def begin(self, iteration: int) -> IterationTransaction:
        if iteration != self.committed_iteration + 1:
            raise ValueError(f"iteration {iteration} does not follow committed {self.committed_iteration}")
        self.cursor.iteration = iteration
        saved = {key: t.detach().clone() for key, t in self._live_buffers().items()}
        self.current = IterationTransaction(iteration, capture_rng_state(), self.cursor.snapshot(), buffers=saved)
        return self.current

    def _step_phase(self, expected: TxnPhase) -> None:
        txn = self.current
        if txn is None or txn.phase is not expected:
            raise RuntimeError(f"transaction not in {expected.value}")
        txn.phase = _NEXT[expected]

    def on_reduced(self) -> None:
        self._step_phase(TxnPhase.COMPUTE)

    def on_step_begin(self) -> None:
        self._step_phase(TxnPhase.REDUCED)

    def on_commit(self) -> None:
        self._step_phase(TxnPhase.STEPPING)
        self._settle(self.current.iteration)

    def _settle(self, iteration: int) -> None:
        """The model now holds the state after ``iteration``; nothing is in flight."""
        self.committed_iteration = iteration
        self.cursor.iteration = iteration + 1
        self.current = None

    @property
    def has_reduced_grads(self) -> bool:
        return self.current is not None and self.current.phase is TxnPhase.REDUCED

    def abort(self) -> dict:
        """Roll the RNG and data cursor back to the start of the in-flight iteration; returns
        the recovery report as it was before the rollback."""
        report = self.recovery_info()
        txn = self.current
        if txn is not None:
            restore_rng_state(txn.rng)
            self.cursor.restore(txn.cursor)
            if txn.phase is not TxnPhase.REDUCED:  # a REDUCED iteration may still roll forward
                txn.phase = TxnPhase.ABORTED
                self._put_back_buffers()
            self.aborts += 1
        return report

    def discard(self) -> None:
        """Drop the in-flight iteration for good (its gradients will not be used)."""
        if self.current is not None:
            self.cursor.restore(self.current.cursor)
            self._put_back_buffers()
        self.current = None

    def adopt(self, iteration: int) -> None:
        """The state was replaced by the state after ``iteration`` (peer copy, snapshot, checkpoint)."""
        self._settle(iteration)

    def recovery_info(self) -> dict:
        inflight = None if self.current is None else self.current.iteration
        return {"committed_iteration": self.committed_iteration, "has_reduced_grads": self.has_reduced_grads,
                "inflight_iteration": inflight}


def roll_forward_plan(recovery: dict[str, dict], world: list[str]) -> dict:
    """The recovery target from the survivors' ABORTED reports: the newest committed iteration.
    ``up_to_date``: ranks already there; ``local_step``: ranks one behind that hold the reduced
    gradients of exactly the target; ``needs_state``: everyone else."""
    blank = {"committed_iteration": -1, "has_reduced_grads": False}
    reports = [(w, recovery.get(w, blank)) for w in world]
    target = max((r.get("committed_iteration", -1) for _, r in reports), default=-1)
    plan = {"target_iteration": target, "local_step": [], "needs_state": [], "up_to_date": []}

    def bucket(r: dict) -> str:
        at = r.get("committed_iteration", -1)
        if at == target:
            return "up_to_date"
        steps_locally = at == target - 1 and r.get("has_reduced_grads") and r.get("inflight_iteration") == target
        return "local_step" if steps_locally else "needs_state"

    for w, r in reports:
        plan[bucket(r)].append(w)
    return plan
