"""The coordinator's worker table: state, incarnation, pid, progress and health of every worker.

A worker that registers again under the same id gets a new incarnation unless it is the same
live process re-announced.  Hang detection reads ``progress_changed_at``: it moves only when the
worker's position ``(gen, iteration, op_seq)`` moves, not on every heartbeat.
Parity: ``resihp/control/membership.py:16-77`` (same record fields, persisted by the coordinator).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from operator import attrgetter


class WorkerState(str, Enum):
    ALIVE = "alive"
    FAILED = "failed"
    FENCED = "fenced"


@dataclass
class WorkerRecord:
    worker_id: str
    node_id: str
    local_rank: int
    device: str = "cpu"
    pid: int = 0
    incarnation: int = 0
    state: WorkerState = WorkerState.ALIVE
    progress: dict = field(default_factory=dict)
    progress_changed_at: float = 0.0
    committed_iteration: int = -1
    has_reduced_grads: bool = False
    health: dict = field(default_factory=dict)

    @property
    def alive(self) -> bool:
        return self.state == WorkerState.ALIVE

    def sort_key(self) -> tuple:
        """Canonical order of workers: node, local rank, id."""
        return self.node_id, self.local_rank, self.worker_id


def _position(progress: dict) -> tuple:
    return progress.get("gen"), progress.get("iteration"), progress.get("op_seq")


class Membership:
    def __init__(self) -> None:
        self.workers: dict[str, WorkerRecord] = {}

    def register(self, rec: WorkerRecord, now: float) -> WorkerRecord:
        earlier = self.workers.get(rec.worker_id)
        if earlier is not None:
            restarted = not (earlier.alive and earlier.pid == rec.pid)
            rec.incarnation = earlier.incarnation + int(restarted)
        rec.progress_changed_at = now
        self.workers[rec.worker_id] = rec
        return rec

    def alive(self) -> list[WorkerRecord]:
        return sorted(filter(attrgetter("alive"), self.workers.values()), key=WorkerRecord.sort_key)

    def alive_ids(self) -> list[str]:
        return list(map(attrgetter("worker_id"), self.alive()))

    def on_node(self, node_id: str) -> list[WorkerRecord]:
        return [rec for rec in self.workers.values() if rec.node_id == node_id]

    def mark(self, worker_ids, state: WorkerState) -> list[str]:
        """Move the live ones among ``worker_ids`` to ``state``; returns those that changed."""
        changed = []
        for wid in worker_ids:
            rec = self.workers.get(wid)
            if rec and rec.alive:
                rec.state = state
                changed.append(wid)
        return changed

    def update_progress(self, worker_id: str, progress: dict, now: float) -> None:
        rec = self.workers.get(worker_id)
        if not (rec and rec.alive):
            return
        if _position(progress) != _position(rec.progress):
            rec.progress_changed_at = now
        rec.progress = progress
        speed = progress.get("p")
        if speed is not None:
            rec.health["p"] = speed
