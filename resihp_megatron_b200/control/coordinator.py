"""Coordinator: the single membership authority of a job.

* Node leases: agents heartbeat for their workers; a node silent for ``lease_timeout`` loses
  all its workers.  Hang detection: when no member of the world made progress for
  ``hang_timeout``, the culprit is a worker not inside a collective, else the one(s) with the
  lowest ``(iteration, op_seq)``.
* Failure declaration and fencing: the agent of a failed worker is told to SIGKILL it, and
  any message of an older generation is ignored.
* Generation-numbered reconfiguration transactions::

      RECONFIG_NOTICE(g) -> ABORTED(g) from every live worker -> planner -> PREPARE(g)
      -> READY(g) from every member of the new world -> COMMIT(g)

  A failure at any point restarts the transaction at g+1, so a crash during a
  reconfiguration is handled like any other crash.  The first transaction skips the notice.
* The data-plane rendezvous store (a c10d ``TCPStore``) lives here, never on a training rank.
* Control state is persisted to a KV store; with ``leader_ttl`` set, replicas elect a leader
  through a KV lease and every write is fenced on still holding the leader key, so a deposed
  leader cannot overwrite its successor.

Behaviour follows the reference's coordinator (``resihp/control/coordinator.py:59-559``);
the transaction is written here as an explicit sequence of phases with one restart point.
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass, field
from typing import Callable

from . import protocol as P
from .kvstore import InMemoryKV, KVStore
from .membership import Membership, WorkerRecord, WorkerState
from ..utils.log import get_logger
from ..utils.rpc import Connection, Server

log = get_logger(__name__)


@dataclass
class ClusterView:
    """What a planner sees: the survivors, what failed, and where the old world was."""

    generation: int
    alive: list[WorkerRecord]
    failed: list[str]
    previous_world: list[str]
    previous_payload: dict | None
    recovery: dict[str, dict]
    reason: str
    reports: dict[str, list[dict]] = field(default_factory=dict)


PlannerFn = Callable[[ClusterView], tuple[list[str], dict]]


def keep_all_planner(view: ClusterView) -> tuple[list[str], dict]:
    world = [w.worker_id for w in view.alive]
    return world, {"world_size": len(world)}


class TransactionRestart(Exception):
    """A failure was declared while a transaction waited; start over at the next generation."""


class Coordinator:
    def __init__(self, *, host: str = "127.0.0.1", port: int = 0, kv: KVStore | None = None,
                 planner: PlannerFn | None = None, expected_workers: int | None = None, min_workers: int = 1,
                 start_grace: float = 5.0, lease_timeout: float = 3.0, hang_timeout: float = 60.0,
                 abort_timeout: float = 15.0, ready_timeout: float = 180.0, host_store: bool = True,
                 store_port: int = 0, namespace: str = "resihp", coordinator_id: str = "coord-0",
                 leader_ttl: float | None = None, tick: float = 0.05,
                 report_handler: Callable[[str, dict], None] | None = None):
        self.host, self._port = host, port
        self.kv: KVStore = kv if kv is not None else InMemoryKV()
        self.planner = planner or keep_all_planner
        self.expected_workers = expected_workers
        self.min_workers = min_workers
        self.start_grace = start_grace
        self.lease_timeout = lease_timeout
        self.hang_timeout = hang_timeout
        self.abort_timeout = abort_timeout
        self.ready_timeout = ready_timeout
        self.host_store = host_store
        self.store_port = store_port
        self.ns = namespace
        self.coordinator_id = coordinator_id
        self.leader_ttl = leader_ttl
        self.tick = tick
        self.report_handler = report_handler

        self.membership = Membership()
        self.generation = 0
        self.committed_generation = 0
        self.world: list[str] = []
        self.payload: dict | None = None
        self.phase = "waiting"
        self.history: list[dict] = []

        self._cv = threading.Condition(threading.RLock())
        self._agents: dict[str, Connection] = {}
        self._node_seen: dict[str, float] = {}
        self._pending_failures: set[str] = set()
        self._failed_since_commit: list[str] = []
        self._planned_reason: str | None = None
        self._force_immediate = False
        self._joiners: set[str] = set()
        self._open_notice: dict | None = None
        self._start_requested = False
        self._first_register: float | None = None
        self._prepared_any = False
        self._aborted: dict[int, dict[str, dict]] = {}
        self._ready: dict[int, set[str]] = {}
        self._build_failed: dict[int, set[str]] = {}
        self._done: set[str] = set()
        self._reports: dict[str, list[dict]] = {}
        self._stopped = threading.Event()
        self._is_leader = threading.Event()
        self._leader_lease: int | None = None
        self.server: Server | None = None
        self.store = None
        self.store_addr: tuple[str, int] | None = None
        self._threads: list[threading.Thread] = []

    # ------------------------------------------------------------------ lifecycle
    @property
    def address(self) -> tuple[str, int]:
        assert self.server is not None, "coordinator not started"
        return self.server.address

    @property
    def is_leader(self) -> bool:
        return self._is_leader.is_set()

    def start(self, block_until_leader: bool = True) -> "Coordinator":
        if self.leader_ttl is None:
            self._become_leader()
        else:
            self._spawn(self._election_loop, "coord-election")
            if block_until_leader:
                self._is_leader.wait()
        return self

    def stop(self) -> None:
        self._stopped.set()
        self._is_leader.clear()
        with self._cv:
            self._cv.notify_all()
        if self.server is not None:
            self.server.stop()
        if self._leader_lease is not None:
            try:
                self.kv.revoke(self._leader_lease)
            except Exception:  # noqa: BLE001
                pass
        self.store = None

    def _spawn(self, fn, name: str) -> None:
        t = threading.Thread(target=fn, name=name, daemon=True)
        t.start()
        self._threads.append(t)

    def _become_leader(self) -> None:
        self._restore_from_kv()
        if self.host_store:
            import torch.distributed as dist  # the control plane itself needs no torch

            self.store = dist.TCPStore(self.host, self.store_port, is_master=True, wait_for_workers=False)
            self.store_addr = (self.host, self.store.port)
        self.server = Server(self.host, self._port, self._on_message, on_close=self._on_conn_close)
        self._is_leader.set()
        self._spawn(self._monitor_loop, "coord-monitor")
        self._spawn(self._reconfig_loop, "coord-reconfig")
        log.warning("%s leads at %s", self.coordinator_id, self.server.address)

    def _election_loop(self) -> None:
        key = f"{self.ns}/leader"
        while not self._stopped.is_set():
            if self._leader_lease is None:
                lease = self.kv.grant_lease(self.leader_ttl)
                if self.kv.cas(key, None, self.coordinator_id, lease=lease):
                    self._leader_lease = lease
                    self._become_leader()
                else:
                    self.kv.revoke(lease)
            elif not self.kv.keepalive(self._leader_lease):
                log.error("%s lost the leader lease", self.coordinator_id)
                self.stop()
                return
            time.sleep(self.leader_ttl / 4)

    # ------------------------------------------------------------------ persistence
    def _snapshot(self) -> dict:
        return {
            "generation": self.generation,
            "committed_generation": self.committed_generation,
            "world": self.world,
            "payload": self.payload,
            "members": {wid: {"node_id": w.node_id, "local_rank": w.local_rank, "device": w.device,
                              "state": w.state.value, "incarnation": w.incarnation, "pid": w.pid,
                              "health": w.health}
                        for wid, w in self.membership.workers.items()},
        }

    def _persist(self) -> bool:
        return self._kv_put(f"{self.ns}/state", json.dumps(self._snapshot()))

    def _kv_put(self, key: str, value: str) -> bool:
        """Fenced write: only while this replica still holds the leader key."""
        if self.leader_ttl is None:
            self.kv.put(key, value)
            return True
        if not self._stopped.is_set() and self.kv.put_if(key, value, f"{self.ns}/leader", self.coordinator_id):
            return True
        if not self._stopped.is_set():
            log.error("%s is no longer the leader; stepping down", self.coordinator_id)
            self._stopped.set()
            self._is_leader.clear()
            threading.Thread(target=self.stop, daemon=True).start()
        return False

    def _restore_from_kv(self) -> None:
        raw = self.kv.get(f"{self.ns}/state")
        if not raw:
            return
        st = json.loads(raw)
        self.generation = st["generation"]
        self.committed_generation = st["committed_generation"]
        self.world = st["world"]
        self.payload = st["payload"]
        # agents need a moment to find the new leader: do not take that for node loss
        grace = time.monotonic() + 2 * self.lease_timeout
        for wid, m in st["members"].items():
            rec = WorkerRecord(worker_id=wid, node_id=m["node_id"], local_rank=m["local_rank"], device=m["device"],
                               pid=m.get("pid", 0), incarnation=m["incarnation"], state=WorkerState(m["state"]),
                               health=dict(m.get("health", {})))
            rec.progress_changed_at = grace
            self.membership.workers[wid] = rec
            if rec.alive:
                self._node_seen[rec.node_id] = grace
        self._prepared_any = self.committed_generation > 0
        self.phase = "running" if self.committed_generation > 0 else "waiting"
        if self.committed_generation > 0 and self.generation > self.committed_generation:
            # predecessor died mid-transaction: workers may sit in PREPARE/READY
            self._planned_reason = "failover"
            self._force_immediate = True
        log.warning("%s restored generation %d (committed %d)", self.coordinator_id, self.generation,
                    self.committed_generation)

    # ------------------------------------------------------------------ messaging
    def _send_to_worker(self, worker_id: str, message: dict) -> bool:
        w = self.membership.workers.get(worker_id)
        conn = self._agents.get(w.node_id) if w is not None else None
        return conn is not None and conn.send(P.msg(P.TO_WORKER, worker_id=worker_id, msg=message))

    def _broadcast(self, worker_ids, message: dict) -> None:
        for wid in worker_ids:
            self._send_to_worker(wid, message)

    def _on_conn_close(self, conn: Connection) -> None:
        node = conn.meta.get("node_id")
        with self._cv:
            if node and self._agents.get(node) is conn:
                del self._agents[node]

    def _on_message(self, conn: Connection, m: dict) -> None:
        kind = m.get("type")
        now = time.monotonic()
        with self._cv:
            if kind == P.AGENT_REGISTER:
                self._on_agent_register(conn, m, now)
            elif kind == P.WORKER_REGISTER:
                self._node_seen[m["node_id"]] = now
                self._register_worker(m, now)
            elif kind == P.NODE_HEARTBEAT:
                if m["node_id"] in self._agents:
                    self._node_seen[m["node_id"]] = now
                for wid, prog in m.get("progress", {}).items():
                    self.membership.update_progress(wid, prog, now)
            elif kind == P.WORKER_FAILED:
                self._declare_failed([m["worker_id"]], m.get("reason", "reported by agent"))
            elif kind == P.WORKER_MSG:
                self._on_worker_message(m["worker_id"], m["msg"])
            self._cv.notify_all()

    def _on_agent_register(self, conn: Connection, m: dict, now: float) -> None:
        node = m["node_id"]
        conn.meta["node_id"] = node
        self._agents[node] = conn
        self._node_seen[node] = now
        for rec in m.get("workers", []):
            self._register_worker(rec, now)
        conn.send(P.msg(P.COORDINATOR_HELLO, coordinator_id=self.coordinator_id, generation=self.generation,
                        committed_generation=self.committed_generation))
        if self._open_notice is not None:  # re-send an open notice the node may have missed
            acked = self._aborted.get(self._open_notice["gen"], {})
            for w in self.membership.on_node(node):
                if w.alive and w.worker_id not in acked:
                    self._send_to_worker(w.worker_id, self._open_notice)

    def _register_worker(self, rec: dict, now: float) -> None:
        wid = rec["worker_id"]
        old = self.membership.workers.get(wid)
        if old is not None and old.alive and old.pid == rec.get("pid", 0):
            return  # same process re-announced by its agent
        if self._first_register is None:
            self._first_register = now
        self.membership.register(WorkerRecord(worker_id=wid, node_id=rec["node_id"],
                                              local_rank=rec.get("local_rank", 0), device=rec.get("device", "cpu"),
                                              pid=rec.get("pid", 0)), now)
        if self.committed_generation > 0 and wid not in self.world:
            self._planned_reason = self._planned_reason or f"join:{wid}"
            self._joiners.add(wid)
        if self._open_notice is not None:
            self._send_to_worker(wid, self._open_notice)
        log.warning("registered %s on %s", wid, rec["node_id"])

    def _on_worker_message(self, worker_id: str, inner: dict) -> None:
        w = self.membership.workers.get(worker_id)
        if w is None or not w.alive:
            return
        kind, gen = inner.get("type"), inner.get("gen", 0)
        if kind == P.ABORTED:
            if gen == self.generation:
                self._aborted.setdefault(gen, {})[worker_id] = inner
                w.committed_iteration = inner.get("committed_iteration", -1)
                w.has_reduced_grads = bool(inner.get("has_reduced_grads", False))
            return
        if kind == P.READY:
            if gen == self.generation:
                self._ready.setdefault(gen, set()).add(worker_id)
            return
        if kind != P.REPORT:
            return
        rkind = inner.get("kind")
        if rkind == "timing":
            if self.report_handler is not None:
                self.report_handler(worker_id, inner)
            return
        self._reports.setdefault(worker_id, []).append(inner)
        if rkind == "build_failed" and inner.get("gen") == self.generation:
            self._build_failed.setdefault(self.generation, set()).add(worker_id)
        elif rkind == "done" and self.phase == "running":
            self._done.add(worker_id)
            if set(self.world) <= self._done:
                self._finish_job()
        elif rkind == "fatal":
            self._declare_failed([worker_id], inner.get("detail", "fatal self-report"))
        elif rkind == "replan" and self.committed_generation > 0:
            self._planned_reason = self._planned_reason or f"replan:{inner.get('detail', '')}"

    # ------------------------------------------------------------------ failures
    def declare_failed(self, worker_ids, reason: str) -> None:
        with self._cv:
            self._declare_failed(worker_ids, reason)
            self._cv.notify_all()

    def _declare_failed(self, worker_ids, reason: str) -> None:
        newly = self.membership.mark(worker_ids, WorkerState.FAILED)
        if not newly or self.phase == "finished":
            return
        log.warning("failed: %s (%s)", newly, reason)
        self.history.append({"t": time.monotonic(), "event": "failure", "workers": newly, "reason": reason})
        for wid in newly:  # fence: the agent SIGKILLs the worker
            conn = self._agents.get(self.membership.workers[wid].node_id)
            if conn is not None:
                conn.send(P.msg(P.KILL, worker_id=wid, reason=reason))
        self._pending_failures.update(newly)
        self._failed_since_commit.extend(newly)

    def _finish_job(self) -> None:
        self.phase = "finished"
        self.history.append({"t": time.monotonic(), "event": "finished", "generation": self.committed_generation})
        self._persist()
        self._broadcast(self.membership.alive_ids(), P.msg(P.SHUTDOWN, gen=self.committed_generation))
        log.warning("job finished at generation %d", self.committed_generation)

    def _mark(self, phase: str, generation: int) -> None:
        self.history.append({"t": time.monotonic(), "event": phase, "generation": generation})

    def request_replan(self, reason: str) -> None:
        with self._cv:
            self._planned_reason = reason
            self._cv.notify_all()

    def set_health(self, worker_id: str, **health) -> None:
        with self._cv:
            w = self.membership.workers.get(worker_id)
            if w is not None:
                w.health.update(health)

    def _monitor_loop(self) -> None:
        while not self._stopped.is_set():
            now = time.monotonic()
            with self._cv:
                for node, seen in list(self._node_seen.items()):
                    if now - seen > self.lease_timeout:
                        victims = [w.worker_id for w in self.membership.on_node(node) if w.alive]
                        if victims:
                            self._declare_failed(victims, f"node {node} lease expired")
                        del self._node_seen[node]
                if self.phase == "running":
                    self._check_hang(now)
                if self.committed_generation == 0 and self.phase == "waiting" and not self._start_requested:
                    self._start_requested = self._ready_to_start(now)
                self._cv.notify_all()
            time.sleep(self.tick)

    def _ready_to_start(self, now: float) -> bool:
        n = len(self.membership.alive())
        if self.expected_workers is not None:
            return n >= self.expected_workers
        return (self._first_register is not None and n >= self.min_workers
                and now - self._first_register >= self.start_grace)

    def _check_hang(self, now: float) -> None:
        members = [w for w in self.membership.alive() if w.worker_id in self.world]
        if not members or any(now - w.progress_changed_at <= self.hang_timeout for w in members):
            return
        suspects = [w for w in members if not w.progress.get("in_collective", False)]
        if not suspects or len(suspects) == len(members):
            def pos(w):
                return (w.progress.get("iteration", -1), w.progress.get("op_seq", -1))

            lowest = min(pos(w) for w in members)
            suspects = [w for w in members if pos(w) == lowest]
        if len(suspects) < len(members):
            self._declare_failed([w.worker_id for w in suspects], "hang (no progress while peers wait)")
        else:
            for w in members:
                w.progress_changed_at = now
            log.error("global stall without an identifiable culprit; extending the deadline")

    # ------------------------------------------------------------------ transactions
    def _reconfig_loop(self) -> None:
        while not self._stopped.is_set():
            with self._cv:
                while not self._stopped.is_set() and not self._has_work():
                    self._cv.wait(self.tick)
                if self._stopped.is_set() or self.phase == "finished":
                    return
                if self._pending_failures:
                    reason = "failure"
                elif self.committed_generation == 0:
                    reason = "start"
                else:
                    reason = self._planned_reason or "replan"
                immediate = bool(self._pending_failures) or self.committed_generation == 0 or self._force_immediate
                self._planned_reason = None
                self._force_immediate = False
                self._start_requested = False
            try:
                self._transaction(reason, immediate)
            except Exception:  # noqa: BLE001 - the authority must not die silently
                log.exception("transaction raised; retrying")
                time.sleep(self.tick)

    def _has_work(self) -> bool:
        return bool(self._pending_failures or self._start_requested
                    or (self._planned_reason and self.committed_generation > 0))

    def _wait(self, pred: Callable[[], bool], timeout: float) -> bool:
        deadline = time.monotonic() + timeout
        with self._cv:
            while not pred():
                if self._pending_failures:
                    raise TransactionRestart()
                left = deadline - time.monotonic()
                if left <= 0 or self._stopped.is_set():
                    return False
                self._cv.wait(min(self.tick, left))
            return True

    def _transaction(self, reason: str, immediate: bool) -> None:
        while not self._stopped.is_set():
            with self._cv:
                self._pending_failures.clear()
                self._done.clear()
                self.generation += 1
                gen = self.generation
                self.phase = "reconfiguring"
                participants = self.membership.alive_ids()
                if not self._persist():
                    return
            try:
                if self._run_phases(gen, reason, immediate, participants):
                    return
                return  # lost leadership / stopped
            except TransactionRestart:
                with self._cv:
                    self._open_notice = None
                reason, immediate = "failure", True

    def _run_phases(self, gen: int, reason: str, immediate: bool, participants: list[str]) -> bool:
        # phase 1: notice + aborted acks (skipped for the very first world)
        if reason == "failover":
            self._wait(lambda: {w.node_id for w in self.membership.alive()} <= set(self._agents),
                       2 * self.lease_timeout)
        if self._prepared_any:
            notice = P.msg(P.RECONFIG_NOTICE, gen=gen, failed=list(self._failed_since_commit), immediate=immediate,
                           reason=reason)
            with self._cv:
                self._open_notice = notice
                self._mark("notice", gen)
            self._broadcast(participants, notice)
            if not self._wait(lambda: set(self.membership.alive_ids()) <= set(self._aborted.get(gen, {})),
                              self.abort_timeout):
                with self._cv:
                    self._open_notice = None
                    silent = sorted(set(self.membership.alive_ids()) - set(self._aborted.get(gen, {})))
                    self._declare_failed(silent, "no ABORTED ack within timeout")
                raise TransactionRestart()
        # phase 2: plan
        with self._cv:
            self._open_notice = None
            self._mark("aborted", gen)
            recovery = dict(self._aborted.get(gen, {}))
            alive = [w for w in self.membership.alive() if not self._prepared_any or w.worker_id in recovery]
            self._joiners -= {w.worker_id for w in alive}
            if not self._joiners and (self._planned_reason or "").startswith("join:"):
                self._planned_reason = None
            view = ClusterView(generation=gen, alive=alive, failed=list(self._failed_since_commit),
                               previous_world=list(self.world), previous_payload=self.payload, recovery=recovery,
                               reason=reason, reports=dict(self._reports))
        world, payload = self.planner(view)
        if not world:
            raise RuntimeError("planner returned an empty world")
        with self._cv:
            self._mark("planned", gen)
            if not (self._persist() and self._kv_put(f"{self.ns}/plan/{gen}",
                                                     json.dumps({"world": world, "payload": payload}))):
                return False
            targets = self.membership.alive_ids()
            self._prepared_any = True
        # phase 3: prepare + ready
        self._broadcast(targets, P.msg(P.PREPARE, gen=gen, world=world, payload=payload, reason=reason,
                                       store_addr=list(self.store_addr) if self.store_addr else None,
                                       store_prefix=f"{self.ns}/gen{gen}/", recovery=recovery))
        if not self._wait(lambda: set(world) <= self._ready.get(gen, set()), self.ready_timeout):
            with self._cv:
                laggards = set(world) - self._ready.get(gen, set())
                # ranks that reported a failed build were blocked by a peer: blame the silent ones
                culprits = (laggards - self._build_failed.get(gen, set())) or laggards
                self._declare_failed(sorted(culprits), "no READY within timeout")
            raise TransactionRestart()
        # phase 4: commit
        with self._cv:
            if self._stopped.is_set():
                return False
            self._mark("ready", gen)
            self.committed_generation = gen
            self.world = list(world)
            self.payload = payload
            self.phase = "running"
            self._failed_since_commit = []
            self._reports = {}
            now = time.monotonic()
            for w in self.membership.alive():
                w.progress_changed_at = now
            if not self._persist():
                return False
            self.history.append({"t": now, "event": "commit", "generation": gen, "world": list(world),
                                 "reason": reason})
            targets = self.membership.alive_ids()
        self._broadcast(targets, P.msg(P.COMMIT, gen=gen))
        log.warning("committed generation %d (%d workers, %s)", gen, len(world), reason)
        return True

    # ------------------------------------------------------------------ introspection
    def wait_for_commit(self, generation: int, timeout: float = 30.0) -> bool:
        deadline = time.monotonic() + timeout
        with self._cv:
            while self.committed_generation < generation:
                left = deadline - time.monotonic()
                if left <= 0:
                    return False
                self._cv.wait(min(0.05, left))
        return True
