"""In-worker control client.

Runs on its own threads (heartbeat + connection reader) and never touches the data plane
except through registered abort callbacks: when a reconfiguration notice arrives while the
training thread is blocked in a collective or a peer-memory kernel, the callbacks raise the
communicator abort (NCCL abort / the device abort word), so the training thread unwinds.

Training-thread API: ``set_progress``, ``set_recovery_info``, ``reconfig_pending``,
``wait_prepare`` (acks a pending notice with ABORTED + recovery info, then blocks for the next
PREPARE), ``send_ready``, ``wait_commit``, ``finish``, ``report``.  Same contract as
``resihp/control/worker_client.py:31-207`` of the reference.
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


class WorkerClient:
    def __init__(self, agent_addr: str | None = None, worker_id: str | None = None, *, local_rank: int | None = None,
                 node_id: str | None = None, device: str | None = None, hb_interval: float = 0.25):
        self.agent_addr = parse_addr(agent_addr or os.environ["RESIHP_AGENT_ADDR"])
        self.worker_id = worker_id or os.environ["RESIHP_WORKER_ID"]
        self.local_rank = local_rank if local_rank is not None else int(os.environ.get("RESIHP_LOCAL_RANK", "0"))
        self.node_id = node_id or os.environ.get("RESIHP_NODE_ID", "node")
        self.device = device or os.environ.get("RESIHP_DEVICE", "cpu")
        self.hb_interval = hb_interval
        self._cv = threading.Condition()
        self._progress: dict = {"gen": 0, "iteration": -1, "op_seq": 0, "phase": "init", "in_collective": False}
        self._recovery: dict = {"committed_iteration": -1, "has_reduced_grads": False}
        self._notice_gen = 0
        self._notice: dict | None = None
        self._acked_gen = 0
        self._prepares: dict[int, dict] = {}
        self._commits: set[int] = set()
        self._in_control_wait = False
        self._abort_callbacks: list[Callable[[], None]] = []
        self._shutdown = False
        self.committed_generation = 0
        self._conn: Connection | None = None
        self._stopped = threading.Event()

    # ------------------------------------------------------------------ lifecycle
    def connect(self, timeout: float = 30.0) -> "WorkerClient":
        self._conn = connect(self.agent_addr, self._on_message, timeout=timeout, name=f"worker-{self.worker_id}")
        self._conn.send(P.msg(P.REGISTER, worker_id=self.worker_id, local_rank=self.local_rank, pid=os.getpid(),
                              device=self.device, node_id=self.node_id))
        threading.Thread(target=self._heartbeat_loop, name="worker-hb", daemon=True).start()
        return self

    def close(self) -> None:
        self._stopped.set()
        if self._conn is not None:
            self._conn.close()

    def _heartbeat_loop(self) -> None:
        while not self._stopped.is_set():
            with self._cv:
                prog = dict(self._progress)
            prog["t"] = time.time()
            if self._conn is not None:
                self._conn.send(P.msg(P.HEARTBEAT, progress=prog))
            time.sleep(self.hb_interval)

    # ------------------------------------------------------------------ training-thread API
    def set_progress(self, **kw) -> None:
        with self._cv:
            if "op_seq" not in kw:
                self._progress["op_seq"] = self._progress.get("op_seq", 0) + 1
            self._progress.update(kw)

    def set_recovery_info(self, **info) -> None:
        with self._cv:
            self._recovery.update(info)

    def add_abort_callback(self, fn: Callable[[], None]) -> None:
        self._abort_callbacks.append(fn)

    def reconfig_pending(self) -> bool:
        with self._cv:
            return self._notice_gen > self.committed_generation

    def immediate_abort_pending(self) -> bool:
        with self._cv:
            return (self._notice_gen > self.committed_generation and self._notice is not None
                    and bool(self._notice.get("immediate")))

    def report(self, kind: str, **detail) -> None:
        if self._conn is not None:
            self._conn.send(P.msg(P.REPORT, kind=kind, **detail))

    def _control_wait(self, pred, timeout: float, what: str):
        """Block (with the notice-ack path enabled) until ``pred()`` returns non-None."""
        deadline = time.monotonic() + timeout
        with self._cv:
            self._in_control_wait = True
            try:
                while True:
                    r = pred()
                    if r is not None:
                        return r
                    left = deadline - time.monotonic()
                    if left <= 0:
                        raise TimeoutError(f"{self.worker_id}: {what}")
                    self._cv.wait(min(0.05, left))
            finally:
                self._in_control_wait = False

    def wait_prepare(self, timeout: float = 600.0) -> dict:
        def pred():
            if self._shutdown:
                raise JobFinished()
            self._ack_locked()
            want = max(self._notice_gen, self.committed_generation + 1)
            ready = [g for g in self._prepares if g >= want]
            if not ready:
                return None
            gen = max(ready)
            for g in [g for g in self._prepares if g < gen]:
                del self._prepares[g]
            return self._prepares[gen]

        return self._control_wait(pred, timeout, "no PREPARE")

    def finish(self, iteration: int, timeout: float = 600.0) -> str:
        """Report completion; returns ``"shutdown"`` when the whole world is done, or
        ``"reconfig"`` if a newer generation needs this worker (e.g. as a state source)."""
        if self._conn is not None:
            self._conn.send(P.msg(P.REPORT, kind="done", iteration=iteration, gen=self.committed_generation))

        def pred():
            if self._shutdown:
                return "shutdown"
            if self._notice_gen > self.committed_generation:
                return "reconfig"
            return None

        return self._control_wait(pred, timeout, "job completion not confirmed")

    @property
    def shutdown(self) -> bool:
        return self._shutdown

    def send_ready(self, gen: int, **info) -> None:
        if self._conn is not None:
            self._conn.send(P.msg(P.READY, gen=gen, **info))

    def wait_commit(self, gen: int, timeout: float = 600.0) -> None:
        def pred():
            if gen in self._commits:
                return True
            if self._notice_gen > gen:
                raise ReconfigInterrupted(f"generation {self._notice_gen} announced while waiting for {gen}")
            return None

        self._control_wait(pred, timeout, f"no COMMIT for generation {gen}")
        with self._cv:
            self.committed_generation = max(self.committed_generation, gen)
            self._progress["gen"] = self.committed_generation

    # ------------------------------------------------------------------ messages
    def _ack_locked(self) -> None:
        if self._notice_gen > self._acked_gen and self._conn is not None:
            self._conn.send(P.msg(P.ABORTED, gen=self._notice_gen, **self._recovery))
            self._acked_gen = self._notice_gen

    def _on_message(self, conn: Connection, m: dict) -> None:
        kind = m.get("type")
        fire: list[Callable[[], None]] = []
        with self._cv:
            if kind == P.RECONFIG_NOTICE:
                if m["gen"] > self._notice_gen:
                    self._notice_gen = m["gen"]
                    self._notice = m
                    if self._in_control_wait:
                        self._ack_locked()
                    elif m.get("immediate", True):
                        fire = list(self._abort_callbacks)
            elif kind == P.SELF_FENCE:
                fire = list(self._abort_callbacks)
            elif kind == P.PREPARE:
                if m["gen"] >= self._notice_gen:
                    self._prepares[m["gen"]] = m
            elif kind == P.COMMIT:
                self._commits.add(m["gen"])
            elif kind == P.SHUTDOWN:
                self._shutdown = True
            self._cv.notify_all()
        for fn in fire:
            try:
                fn()
            except Exception:  # noqa: BLE001 - abort is best effort; the waiter times out otherwise
                log.exception("abort callback raised")
