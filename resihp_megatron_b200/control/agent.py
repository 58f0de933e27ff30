"""NodeAgent: one per node, between the node's workers and the coordinator.

* Starts (or adopts) the node's workers and never tears healthy ones down when a peer dies --
  the opposite of an elastic launcher that restarts everybody.
* Folds the workers' heartbeats into one node heartbeat, so the coordinator's load grows with
  nodes, not GPUs.
* Notices local deaths at once -- process exit, a lost control connection, a heartbeat that
  stalled (a hang), a fatal health event -- and reports them.
* Fences on command: SIGKILL of a worker the coordinator declared failed.
* Fails over between coordinator replicas; after ``self_fence_after`` seconds with no
  coordinator at all it tells its workers to self-fence (abort their communicators).
Parity: ``resihp/control/agent.py:59-265`` (same duties, messages and environment variables).
"""

from __future__ import annotations

import contextlib
import os
import signal
import subprocess
import threading
import time
from dataclasses import dataclass, field

from . import protocol as P
from ..utils.log import get_logger
from ..utils.rpc import Connection, Server, connect, fmt_addr

log = get_logger(__name__)


def pid_alive(pid: int) -> bool:
    """Whether ``pid`` still runs (a zombie child of this process counts as gone)."""
    if pid <= 0:
        return False
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True  # exists, owned by someone else
    try:
        reaped, _status = os.waitpid(pid, os.WNOHANG)
    except ChildProcessError:
        return True  # not our child: existence is all we can know
    return reaped == 0


PF_EXITING = 0x4  # Linux task flag: the task has entered exit (set before its memory is torn down)


def parse_stat_exiting(stat: str) -> bool:
    """``/proc/<pid>/stat`` text -> whether the task is exiting or already a zombie / dead.  The
    command name is parenthesised and may itself contain spaces or parentheses, so the fields are
    taken after the last ``)``: state, ppid, pgrp, session, tty, tpgid, flags, ..."""
    rest = stat[stat.rfind(")") + 2:].split()
    if len(rest) < 7:
        return False
    return rest[0] in ("Z", "X", "x") or bool(int(rest[6]) & PF_EXITING)


def pid_exiting(pid: int) -> bool:
    """Whether ``pid`` has started to exit (Linux).  A SIGKILLed GPU process can take a few hundred
    milliseconds between this point and the closing of its sockets -- the driver unmaps its device
    memory first -- so this sees a dead worker well before its control connection drops."""
    if pid <= 0:
        return False
    try:
        with open(f"/proc/{pid}/stat", encoding="ascii", errors="replace") as fh:
            return parse_stat_exiting(fh.read())
    except (OSError, ValueError):
        return False


@dataclass
class LocalWorker:
    worker_id: str
    local_rank: int
    pid: int = 0
    device: str = "cpu"
    proc: subprocess.Popen | None = None
    conn: Connection | None = None
    last_hb: float = field(default_factory=time.monotonic)
    progress: dict = field(default_factory=dict)
    dead: bool = False

    def death_reason(self, now: float, stall_after: float) -> str | None:
        code = self.proc.poll() if self.proc is not None else None
        if code is not None:
            return f"exited with {code}"
        if self.proc is None and self.pid and not pid_alive(self.pid):
            return "process gone"
        if self.pid and pid_exiting(self.pid):
            return "process exiting"
        silent = now - self.last_hb
        if self.conn is not None and silent > stall_after:
            return f"heartbeat stalled {silent:.1f}s (hang)"
        return None


class _Uplink:
    """The agent's link to the current coordinator replica."""

    def __init__(self, agent: "NodeAgent", addrs):
        self.agent, self.addrs = agent, list(addrs)
        self.conn: Connection | None = None
        self.lost_at: float | None = None
        self.fenced = False

    def send(self, message: dict) -> None:
        link = self.conn
        if link is None or not link.send(message):
            log.warning("no coordinator; dropped %s", message.get("type"))

    def dial(self, timeout: float) -> bool:
        """Try every replica until one answers (or ``timeout``), then register this node."""
        a = self.agent
        give_up = time.monotonic() + timeout
        while time.monotonic() < give_up and not a._stopped.is_set():
            for addr in self.addrs:
                try:
                    link = connect(addr, a._from_coordinator, self._closed, timeout=0.5, name=f"agent-{a.node_id}")
                except TimeoutError:
                    continue
                with a._lock:
                    self.conn, self.lost_at, self.fenced = link, None, False
                    known = [dict(worker_id=w.worker_id, node_id=a.node_id, local_rank=w.local_rank, pid=w.pid,
                                  device=w.device) for w in a.workers.values() if not w.dead and w.conn is not None]
                link.send(P.msg(P.AGENT_REGISTER, node_id=a.node_id, workers=known))
                return True
            time.sleep(0.1)
        return False

    def _closed(self, conn: Connection) -> None:
        with self.agent._lock:
            if self.conn is conn:
                self.conn, self.lost_at = None, time.monotonic()

    def overdue(self, after: float) -> bool:
        """True once per outage, when no coordinator has answered for ``after`` seconds."""
        since = self.lost_at if self.lost_at is not None else time.monotonic()
        if self.fenced or time.monotonic() - since <= after:
            return False
        self.fenced = True
        return True


class NodeAgent:
    def __init__(self, node_id: str, coordinator_addrs: list[tuple[str, int]], *, host: str = "127.0.0.1",
                 port: int = 0, hb_interval: float = 0.25, worker_timeout: float = 2.0,
                 self_fence_after: float = 5.0, health_probe=None, health_every: int = 8):
        self.node_id = node_id
        self.coordinator_addrs = list(coordinator_addrs)
        self.hb_interval, self.worker_timeout, self.self_fence_after = hb_interval, worker_timeout, self_fence_after
        self.health_probe, self.health_every = health_probe, health_every
        self.workers: dict[str, LocalWorker] = {}
        self._lock = threading.RLock()
        self._stopped = threading.Event()
        self._up = _Uplink(self, coordinator_addrs)
        self.server = Server(host, port, self._from_worker, on_close=self._worker_link_closed)
        self._threads: list[threading.Thread] = []

    @property
    def address(self) -> tuple[str, int]:
        return self.server.address

    def start(self) -> "NodeAgent":
        self._up.dial(timeout=10.0)
        for loop, name in ((self._beat, "agent-hb"), (self._sweep, "agent-monitor")):
            t = threading.Thread(target=loop, name=f"{name}-{self.node_id}", daemon=True)
            self._threads.append(t)
            t.start()
        return self

    def stop(self, kill_workers: bool = False) -> None:
        self._stopped.set()
        if kill_workers:
            for w in list(self.workers.values()):
                self._sigkill(w)
        if self._up.conn is not None:
            self._up.conn.close()
        self.server.stop()

    # ------------------------------------------------------------------ processes
    def spawn(self, cmd: list[str], nproc: int, env: dict[str, str] | None = None,
              devices: list[str] | None = None, first_rank: int = 0) -> list[LocalWorker]:
        """Start ``nproc`` workers with local ranks ``first_rank, first_rank + 1, ...``; each learns
        its identity from ``RESIHP_*`` variables (and its GPU from ``CUDA_VISIBLE_DEVICES``).  A
        later call with a higher ``first_rank`` adds workers to a running job -- a replacement GPU,
        a grown node -- which register and join at the next generation."""
        launched = []
        for k in range(nproc):
            rank = first_rank + k
            device = devices[k] if devices else "cpu"
            wid = f"{self.node_id}g{rank}"
            child_env = dict(os.environ)
            child_env.update(env or {})
            child_env.update(RESIHP_AGENT_ADDR=fmt_addr(self.address), RESIHP_WORKER_ID=wid,
                             RESIHP_NODE_ID=self.node_id, RESIHP_LOCAL_RANK=str(rank), RESIHP_DEVICE=device)
            if device.startswith("cuda:"):
                child_env["CUDA_VISIBLE_DEVICES"] = device.partition(":")[2]
            proc = subprocess.Popen(cmd, env=child_env)
            w = LocalWorker(wid, rank, pid=proc.pid, device=device, proc=proc)
            with self._lock:
                self.workers[wid] = w
            launched.append(w)
        return launched

    def _sigkill(self, w: LocalWorker) -> None:
        if w.pid > 0:
            with contextlib.suppress(ProcessLookupError):
                os.kill(w.pid, signal.SIGKILL)
        if w.proc is not None:
            with contextlib.suppress(subprocess.TimeoutExpired):
                w.proc.wait(timeout=5)

    def _declare_dead(self, w: LocalWorker, reason: str) -> None:
        if not w.dead:
            w.dead = True
            log.warning("worker %s dead: %s", w.worker_id, reason)
            self._up.send(P.msg(P.WORKER_FAILED, worker_id=w.worker_id, node_id=self.node_id, reason=reason))

    # ------------------------------------------------------------------ worker side
    def _from_worker(self, conn: Connection, m: dict) -> None:
        if m.get("type") == P.REGISTER:
            self._adopt(conn, m)
            return
        with self._lock:
            w = self.workers.get(conn.meta.get("worker_id"))
            if w is None or w.dead:
                return
            w.last_hb = time.monotonic()
            if m.get("type") == P.HEARTBEAT:
                w.progress = m.get("progress", {})
                return
        self._up.send(P.msg(P.WORKER_MSG, worker_id=w.worker_id, msg=m))

    def _adopt(self, conn: Connection, m: dict) -> None:
        wid = m["worker_id"]
        with self._lock:
            w = self.workers.get(wid)
            if w is None or w.dead:  # a worker this agent did not start (or a restarted one)
                w = self.workers[wid] = LocalWorker(wid, m.get("local_rank", 0))
            w.pid, w.device = m.get("pid", w.pid), m.get("device", w.device)
            w.conn, w.last_hb = conn, time.monotonic()
            conn.meta["worker_id"] = wid
        self._up.send(P.msg(P.WORKER_REGISTER, worker_id=wid, node_id=self.node_id, local_rank=w.local_rank,
                            pid=w.pid, device=w.device))

    def _worker_link_closed(self, conn: Connection) -> None:
        wid = conn.meta.get("worker_id")
        if wid is None or self._stopped.is_set():
            return
        with self._lock:
            w = self.workers.get(wid)
            if w is not None and w.conn is conn:
                self._declare_dead(w, "control connection lost")

    def _sweep(self) -> None:
        """Liveness of every local worker, and (every ``health_every`` sweeps) the health probe."""
        sweeps = 0
        while not self._stopped.is_set():
            now = time.monotonic()
            with self._lock:
                for w in [w for w in self.workers.values() if not w.dead]:
                    why = w.death_reason(now, self.worker_timeout)
                    if why is not None:
                        self._declare_dead(w, why)
            sweeps += 1
            if self.health_probe is not None and sweeps % self.health_every == 0:
                self._apply_health(self.health_probe.poll())
            time.sleep(self.hb_interval / 2)

    def _apply_health(self, events) -> None:
        for ev in filter(lambda e: e.fatal, events):
            with self._lock:
                for w in self.workers.values():
                    if not w.dead and ev.matches(w.device):
                        self._declare_dead(w, f"health: {ev.describe()}")

    # ------------------------------------------------------------------ coordinator side
    def _from_coordinator(self, conn: Connection, m: dict) -> None:
        kind = m.get("type")
        if kind not in (P.KILL, P.TO_WORKER):
            return
        with self._lock:
            w = self.workers.get(m["worker_id"])
        if w is None:
            return
        if kind == P.KILL:
            log.warning("fencing %s: %s", w.worker_id, m.get("reason"))
            w.dead = True
            self._sigkill(w)
        elif not w.dead and w.conn is not None:
            w.conn.send(m["msg"])

    def _beat(self) -> None:
        while not self._stopped.is_set():
            if self._up.conn is not None:
                with self._lock:
                    snapshot = {w.worker_id: w.progress for w in self.workers.values() if not w.dead}
                self._up.send(P.msg(P.NODE_HEARTBEAT, node_id=self.node_id, progress=snapshot))
            else:
                if self._up.overdue(self.self_fence_after):
                    with self._lock:
                        for w in self.workers.values():
                            if not w.dead and w.conn is not None:
                                w.conn.send(P.msg(P.SELF_FENCE, reason="coordinator unreachable"))
                self._up.dial(timeout=self.hb_interval)
            time.sleep(self.hb_interval)
