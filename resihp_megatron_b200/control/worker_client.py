"""The control client inside a worker process.

It runs on its own threads (heartbeat, connection reader) and touches the data plane only
through registered abort callbacks: when a reconfiguration notice arrives while the training
thread is blocked in a collective or a peer-memory kernel, the callbacks abort the
communicators (NCCL abort, the device abort word) so the training thread unwinds.

Training-thread API: ``set_progress``, ``set_recovery_info``, ``reconfig_pending``,
``wait_prepare`` (acknowledges a pending notice with ABORTED and the recovery info, then blocks
for the next PREPARE), ``send_ready``, ``wait_commit``, ``finish`` and ``report``.
Parity: ``resihp/control/worker_client.py:31-207`` (same contract and messages).
"""

from __future__ import annotations

import os
import threading
import time
from typing import Callable

from . import protocol as P
from ..utils.log import get_logger
from ..utils.rpc import Connection, connect, parse_addr

log = get_logger(__name__)


class ReconfigInterrupted(Exception):
    """A newer generation was announced while this worker waited on an older one."""


class JobFinished(Exception):
    """The coordinator declared the job complete."""


def _env(name: str, default=None):
    return os.environ.get(name, default)


class WorkerClient:
    def __init__(self, agent_addr: str | None = None, worker_id: str | None = None, *, local_rank: int | None = None,
                 node_id: str | None = None, device: str | None = None, hb_interval: float = 0.25):
        self.agent_addr = parse_addr(agent_addr or os.environ["RESIHP_AGENT_ADDR"])
        self.worker_id = worker_id or os.environ["RESIHP_WORKER_ID"]
        self.local_rank = int(_env("RESIHP_LOCAL_RANK", "0")) if local_rank is None else local_rank
        self.node_id = node_id or _env("RESIHP_NODE_ID", "node")
        self.device = device or _env("RESIHP_DEVICE", "cpu")
        self.hb_interval = hb_interval
        self.committed_generation = 0
        self._cv = threading.Condition()
        self._progress = dict(gen=0, iteration=-1, op_seq=0, phase="init", in_collective=False)
        self._recovery = dict(committed_iteration=-1, has_reduced_grads=False)
        self._latest_notice: dict | None = None   # the newest RECONFIG_NOTICE
        self._acked = 0                            # generation of the last ABORTED sent
        self._prepared: dict[int, dict] = {}       # generation -> PREPARE
        self._committed: set[int] = set()
        self._blocked_in_control = False
        self._abort_hooks: list[Callable[[], None]] = []
        self._shutdown = False
        self._conn: Connection | None = None
        self._stopped = threading.Event()
        # arrival time (time.monotonic, machine-wide) of every notice / PREPARE, by generation
        self.arrivals: dict[str, float] = {}
        self._handlers = {P.RECONFIG_NOTICE: self._got_notice, P.SELF_FENCE: self._got_self_fence,
                          P.PREPARE: self._got_prepare, P.COMMIT: self._got_commit, P.SHUTDOWN: self._got_shutdown}

    @property
    def _notice_gen(self) -> int:
        return self._latest_notice["gen"] if self._latest_notice is not None else 0

    # ------------------------------------------------------------------ lifecycle
    def connect(self, timeout: float = 30.0) -> "WorkerClient":
        self._conn = connect(self.agent_addr, self._on_message, timeout=timeout, name=f"worker-{self.worker_id}")
        self._send(P.msg(P.REGISTER, worker_id=self.worker_id, local_rank=self.local_rank, pid=os.getpid(),
                         device=self.device, node_id=self.node_id))
        threading.Thread(target=self._heartbeats, name="worker-hb", daemon=True).start()
        return self

    def close(self) -> None:
        self._stopped.set()
        if self._conn is not None:
            self._conn.close()

    def _send(self, message: dict) -> None:
        if self._conn is not None:
            self._conn.send(message)

    def _heartbeats(self) -> None:
        while not self._stopped.is_set():
            with self._cv:
                snapshot = {**self._progress, "t": time.time()}
            self._send(P.msg(P.HEARTBEAT, progress=snapshot))
            time.sleep(self.hb_interval)

    # ------------------------------------------------------------------ training-thread API
    def set_progress(self, **kw) -> None:
        """Update the reported position; every call without ``op_seq`` advances it by one."""
        with self._cv:
            kw.setdefault("op_seq", self._progress.get("op_seq", 0) + 1)
            self._progress.update(kw)

    def set_recovery_info(self, **info) -> None:
        with self._cv:
            self._recovery.update(info)

    def add_abort_callback(self, fn: Callable[[], None]) -> None:
        self._abort_hooks.append(fn)

    def reconfig_pending(self) -> bool:
        with self._cv:
            return self._notice_gen > self.committed_generation

    def immediate_abort_pending(self) -> bool:
        with self._cv:
            pending = self._notice_gen > self.committed_generation
            return pending and bool(self._latest_notice.get("immediate"))

    @property
    def shutdown(self) -> bool:
        return self._shutdown

    def report(self, kind: str, **detail) -> None:
        self._send(P.msg(P.REPORT, kind=kind, **detail))

    def send_ready(self, gen: int, **info) -> None:
        self._send(P.msg(P.READY, gen=gen, **info))

    def _block(self, check: Callable[[], object], timeout: float, what: str):
        """Wait until ``check()`` returns something other than None (it may raise).  While the
        training thread sits here, a new notice is acknowledged straight away."""
        deadline = time.monotonic() + timeout
        with self._cv:
            self._blocked_in_control = True
            try:
                while (answer := check()) is None:
                    remaining = deadline - time.monotonic()
                    if remaining <= 0:
                        raise TimeoutError(f"{self.worker_id}: {what}")
                    self._cv.wait(min(0.05, remaining))
                return answer
            finally:
                self._blocked_in_control = False

    def wait_prepare(self, timeout: float = 600.0) -> dict:
        def newest_prepare():
            if self._shutdown:
                raise JobFinished()
            self._acknowledge()
            floor = max(self._notice_gen, self.committed_generation + 1)
            fresh = [g for g in self._prepared if g >= floor]
            if not fresh:
                return None
            top = max(fresh)
            self._prepared = {g: m for g, m in self._prepared.items() if g >= top}
            return self._prepared[top]

        return self._block(newest_prepare, timeout, "no PREPARE")

    def finish(self, iteration: int, timeout: float = 600.0) -> str:
        """Report this worker done; returns ``"shutdown"`` once the whole world is done, or
        ``"reconfig"`` when a newer generation still needs it (e.g. as a state source)."""
        self._send(P.msg(P.REPORT, kind="done", iteration=iteration, gen=self.committed_generation))

        def outcome():
            if self._shutdown:
                return "shutdown"
            return "reconfig" if self._notice_gen > self.committed_generation else None

        return self._block(outcome, timeout, "job completion not confirmed")

    def wait_commit(self, gen: int, timeout: float = 600.0) -> None:
        def committed():
            if gen in self._committed:
                return True
            if self._notice_gen > gen:
                raise ReconfigInterrupted(f"generation {self._notice_gen} announced while waiting for {gen}")
            return None

        self._block(committed, timeout, f"no COMMIT for generation {gen}")
        with self._cv:
            self.committed_generation = max(gen, self.committed_generation)
            self._progress["gen"] = self.committed_generation

    # ------------------------------------------------------------------ incoming messages (reader thread)
    def _acknowledge(self) -> None:
        gen = self._notice_gen
        if gen > self._acked and self._conn is not None:
            self._conn.send(P.msg(P.ABORTED, gen=gen, **self._recovery))
            self._acked = gen

    def _got_notice(self, m: dict) -> list:
        if m["gen"] <= self._notice_gen:
            return []
        self._latest_notice = m
        self.arrivals[f"notice{m['gen']}"] = time.monotonic()
        if self._blocked_in_control:
            self._acknowledge()
            return []
        return list(self._abort_hooks) if m.get("immediate", True) else []

    def _got_self_fence(self, m: dict) -> list:
        return list(self._abort_hooks)

    def _got_prepare(self, m: dict) -> list:
        if m["gen"] >= self._notice_gen:
            self._prepared[m["gen"]] = m
            self.arrivals[f"prepare{m['gen']}"] = time.monotonic()
        return []

    def _got_commit(self, m: dict) -> list:
        self._committed.add(m["gen"])
        return []

    def _got_shutdown(self, m: dict) -> list:
        self._shutdown = True
        return []

    def _on_message(self, conn: Connection, m: dict) -> None:
        handler = self._handlers.get(m.get("type"))
        with self._cv:
            hooks = handler(m) if handler is not None else []
            self._cv.notify_all()
        for hook in hooks:  # outside the lock: an abort may block briefly
            try:
                hook()
            except Exception:  # noqa: BLE001 -- best effort; a waiter times out otherwise
                log.exception("abort callback raised")
