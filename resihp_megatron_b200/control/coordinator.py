"""Coordinator: the one membership authority of a job.

Responsibilities

* **Liveness.**  Agents heartbeat for their node's workers; a node silent for ``lease_timeout``
  loses all of them.  A hang is declared when no member of the world made progress for
  ``hang_timeout``: the culprits are the members not inside a collective, or else the ones
  furthest behind in ``(iteration, op_seq)``.
* **Fencing.**  A failed worker's agent is told to SIGKILL it, and every message of an older
  generation is dropped.
* **Reconfiguration transactions**, one generation each::

      RECONFIG_NOTICE(g) -> ABORTED(g) from every live worker -> planner -> PREPARE(g)
      -> READY(g) from every member of the new world -> COMMIT(g)

  A failure declared while a transaction waits restarts it at ``g + 1``, so a crash during a
  reconfiguration is handled like any other.  The first world skips the notice.
* **Rendezvous.**  The data plane's c10d ``TCPStore`` lives here, never on a training rank;
  generation ``g`` uses the key prefix ``{ns}/gen{g}/``.
* **State and HA.**  Control state is written to a KV store (``{ns}/state``,
  ``{ns}/plan/{g}``).  With ``leader_ttl``, replicas elect a leader through a lease on
  ``{ns}/leader`` and every write is fenced on still holding it, so a deposed leader can never
  overwrite its successor; a new leader resumes from the stored state, including a transaction
  its predecessor left open.

Parity: ``resihp/control/coordinator.py:59-559`` (same protocol, KV keys and semantics).  Here
the message handling is a dispatch table, acknowledgements live in a per-generation ledger,
leadership in its own helper, and one transaction attempt is an object with four steps.
"""

from __future__ import annotations

import json
import threading
import time
from collections import defaultdict
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
    """What a planner sees: the survivors, what failed, and the world it replaces."""

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
    """A failure was declared while a transaction waited: start over at the next generation."""


class _Ledger:
    """Acknowledgements per generation: ABORTED payloads, READY senders, failed builds."""

    def __init__(self):
        self.aborted: dict[int, dict[str, dict]] = defaultdict(dict)
        self.ready: dict[int, set[str]] = defaultdict(set)
        self.build_failed: dict[int, set[str]] = defaultdict(set)


class _Leadership:
    """Leader election on ``{ns}/leader`` and fenced KV writes."""

    def __init__(self, coord: "Coordinator"):
        self.c = coord
        self.lease: int | None = None
        self.key = f"{coord.ns}/leader"

    def write(self, key: str, value: str) -> bool:
        c = self.c
        if c.leader_ttl is None:
            c.kv.put(key, value)
            return True
        if not c._stopped.is_set() and c.kv.put_if(key, value, self.key, c.coordinator_id):
            return True
        if not c._stopped.is_set():
            log.error("%s is no longer the leader; stepping down", c.coordinator_id)
            c._stopped.set()
            c._is_leader.clear()
            threading.Thread(target=c.stop, daemon=True).start()
        return False

    def campaign(self) -> None:
        c = self.c
        while not c._stopped.is_set():
            if self.lease is not None:
                if not c.kv.keepalive(self.lease):
                    log.error("%s lost the leader lease", c.coordinator_id)
                    c.stop()
                    return
            else:
                lease = c.kv.grant_lease(c.leader_ttl)
                if c.kv.cas(self.key, None, c.coordinator_id, lease=lease):
                    self.lease = lease
                    c._become_leader()
                else:
                    c.kv.revoke(lease)
            time.sleep(c.leader_ttl / 4)

    def release(self) -> None:
        if self.lease is not None:
            try:
                self.c.kv.revoke(self.lease)
            except Exception:  # noqa: BLE001
                pass


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
        self.expected_workers, self.min_workers, self.start_grace = expected_workers, min_workers, start_grace
        self.lease_timeout, self.hang_timeout = lease_timeout, hang_timeout
        self.abort_timeout, self.ready_timeout = abort_timeout, ready_timeout
        self.host_store, self.store_port = host_store, store_port
        self.ns, self.coordinator_id, self.leader_ttl = namespace, coordinator_id, leader_ttl
        self.tick = tick
        self.report_handler = report_handler

        # public state
        self.membership = Membership()
        self.generation = 0
        self.committed_generation = 0
        self.world: list[str] = []
        self.payload: dict | None = None
        self.phase = "waiting"
        self.history: list[dict] = []
        self.server: Server | None = None
        self.store = None
        self.store_addr: tuple[str, int] | None = None

        self._cv = threading.Condition(threading.RLock())
        self._stopped = threading.Event()
        self._is_leader = threading.Event()
        self._lead = _Leadership(self)
        self._ledger = _Ledger()
        self._agents: dict[str, Connection] = {}
        self._node_seen: dict[str, float] = {}
        self._failures: set[str] = set()          # declared, not yet handled by a transaction
        self._failed_since_commit: list[str] = []
        self._replan_reason: str | None = None
        self._force_immediate = False
        self._joiners: set[str] = set()
        self._open_notice: dict | None = None
        self._start_requested = False
        self._first_register: float | None = None
        self._prepared_any = False
        self._done: set[str] = set()
        self._reports: dict[str, list[dict]] = defaultdict(list)
        self._threads: list[threading.Thread] = []
        self._on = {P.AGENT_REGISTER: self._agent_register, P.WORKER_REGISTER: self._worker_register_msg,
                    P.NODE_HEARTBEAT: self._node_heartbeat, P.WORKER_FAILED: self._worker_failed,
                    P.WORKER_MSG: self._worker_msg}
        self._on_report = {"build_failed": self._report_build_failed, "done": self._report_done,
                           "fatal": self._report_fatal, "replan": self._report_replan}

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
            return self
        self._thread(self._lead.campaign, "coord-election")
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
        self._lead.release()
        self.store = None

    def _thread(self, fn, name: str) -> None:
        t = threading.Thread(target=fn, name=name, daemon=True)
        self._threads.append(t)
        t.start()

    def _become_leader(self) -> None:
        self._restore()
        if self.host_store:
            import torch.distributed as dist  # the control plane itself needs no torch

            self.store = dist.TCPStore(self.host, self.store_port, is_master=True, wait_for_workers=False)
            self.store_addr = (self.host, self.store.port)
        self.server = Server(self.host, self._port, self._dispatch, on_close=self._agent_gone)
        self._is_leader.set()
        self._thread(self._watch, "coord-monitor")
        self._thread(self._drive, "coord-reconfig")
        log.warning("%s leads at %s", self.coordinator_id, self.server.address)

    # ------------------------------------------------------------------ persisted state
    def _state_json(self) -> str:
        members = {wid: dict(node_id=w.node_id, local_rank=w.local_rank, device=w.device, state=w.state.value,
                             incarnation=w.incarnation, pid=w.pid, health=w.health)
                   for wid, w in self.membership.workers.items()}
        return json.dumps(dict(generation=self.generation, committed_generation=self.committed_generation,
                               world=self.world, payload=self.payload, members=members))

    def _persist(self) -> bool:
        return self._lead.write(f"{self.ns}/state", self._state_json())

    def _restore(self) -> None:
        raw = self.kv.get(f"{self.ns}/state")
        if not raw:
            return
        saved = json.loads(raw)
        self.generation, self.committed_generation = saved["generation"], saved["committed_generation"]
        self.world, self.payload = saved["world"], saved["payload"]
        # agents need a moment to find a new leader: do not mistake that for a node loss
        settle = time.monotonic() + 2 * self.lease_timeout
        for wid, m in saved["members"].items():
            rec = WorkerRecord(wid, m["node_id"], m["local_rank"], device=m["device"], pid=m.get("pid", 0),
                               incarnation=m["incarnation"], state=WorkerState(m["state"]),
                               health=dict(m.get("health", {})), progress_changed_at=settle)
            self.membership.workers[wid] = rec
            if rec.alive:
                self._node_seen[rec.node_id] = settle
        running = self.committed_generation > 0
        self._prepared_any, self.phase = running, ("running" if running else "waiting")
        if running and self.generation > self.committed_generation:
            # the predecessor died inside a transaction: workers may be waiting in PREPARE/READY
            self._replan_reason, self._force_immediate = "failover", True
        log.warning("%s restored generation %d (committed %d)", self.coordinator_id, self.generation,
                    self.committed_generation)

    # ------------------------------------------------------------------ messages
    def _to_worker(self, worker_id: str, message: dict) -> bool:
        rec = self.membership.workers.get(worker_id)
        link = self._agents.get(rec.node_id) if rec else None
        return bool(link) and link.send(P.msg(P.TO_WORKER, worker_id=worker_id, msg=message))

    def _broadcast(self, worker_ids, message: dict) -> None:
        for wid in worker_ids:
            self._to_worker(wid, message)

    def _agent_gone(self, conn: Connection) -> None:
        node = conn.meta.get("node_id")
        with self._cv:
            if node is not None and self._agents.get(node) is conn:
                self._agents.pop(node)

    def _dispatch(self, conn: Connection, m: dict) -> None:
        handler = self._on.get(m.get("type"))
        with self._cv:
            if handler is not None:
                handler(conn, m, time.monotonic())
            self._cv.notify_all()

    def _agent_register(self, conn: Connection, m: dict, now: float) -> None:
        node = m["node_id"]
        conn.meta["node_id"] = node
        self._agents[node] = conn
        self._node_seen[node] = now
        for rec in m.get("workers", []):
            self._register(rec, now)
        conn.send(P.msg(P.COORDINATOR_HELLO, coordinator_id=self.coordinator_id, generation=self.generation,
                        committed_generation=self.committed_generation))
        notice = self._open_notice
        if notice is not None:  # the node may have missed it while it was reconnecting
            acked = self._ledger.aborted[notice["gen"]]
            self._broadcast([w.worker_id for w in self.membership.on_node(node)
                             if w.alive and w.worker_id not in acked], notice)

    def _worker_register_msg(self, conn: Connection, m: dict, now: float) -> None:
        self._node_seen[m["node_id"]] = now
        self._register(m, now)

    def _node_heartbeat(self, conn: Connection, m: dict, now: float) -> None:
        if m["node_id"] in self._agents:
            self._node_seen[m["node_id"]] = now
        for wid, progress in m.get("progress", {}).items():
            self.membership.update_progress(wid, progress, now)

    def _worker_failed(self, conn: Connection, m: dict, now: float) -> None:
        self._declare_failed([m["worker_id"]], m.get("reason", "reported by agent"))

    def _register(self, rec: dict, now: float) -> None:
        wid = rec["worker_id"]
        known = self.membership.workers.get(wid)
        if known is not None and known.alive and known.pid == rec.get("pid", 0):
            return  # the same process, re-announced by its agent after a reconnect
        self._first_register = self._first_register or now
        self.membership.register(WorkerRecord(wid, rec["node_id"], rec.get("local_rank", 0),
                                              device=rec.get("device", "cpu"), pid=rec.get("pid", 0)), now)
        if self.committed_generation > 0 and wid not in self.world:
            self._joiners.add(wid)
            self._replan_reason = self._replan_reason or f"join:{wid}"
        if self._open_notice is not None:
            self._to_worker(wid, self._open_notice)
        log.warning("registered %s on %s", wid, rec["node_id"])

    def _worker_msg(self, conn: Connection, m: dict, now: float) -> None:
        wid, inner = m["worker_id"], m["msg"]
        rec = self.membership.workers.get(wid)
        if rec is None or not rec.alive:
            return
        kind, gen = inner.get("type"), inner.get("gen", 0)
        if kind == P.ABORTED and gen == self.generation:
            self._ledger.aborted[gen][wid] = inner
            rec.committed_iteration = inner.get("committed_iteration", -1)
            rec.has_reduced_grads = bool(inner.get("has_reduced_grads", False))
        elif kind == P.READY and gen == self.generation:
            self._ledger.ready[gen].add(wid)
        elif kind == P.REPORT:
            self._report(wid, inner)

    def _report(self, wid: str, report: dict) -> None:
        kind = report.get("kind")
        if kind == "timing":
            if self.report_handler is not None:
                self.report_handler(wid, report)
            return
        self._reports[wid].append(report)
        handler = self._on_report.get(kind)
        if handler is not None:
            handler(wid, report)

    def _report_build_failed(self, wid: str, report: dict) -> None:
        if report.get("gen") == self.generation:
            self._ledger.build_failed[self.generation].add(wid)

    def _report_done(self, wid: str, report: dict) -> None:
        if self.phase != "running":
            return
        self._done.add(wid)
        if self._done.issuperset(self.world):
            self._finish_job()

    def _report_fatal(self, wid: str, report: dict) -> None:
        self._declare_failed([wid], report.get("detail", "fatal self-report"))

    def _report_replan(self, wid: str, report: dict) -> None:
        if self.committed_generation > 0:
            self._replan_reason = self._replan_reason or f"replan:{report.get('detail', '')}"

    # ------------------------------------------------------------------ failures and requests
    def declare_failed(self, worker_ids, reason: str) -> None:
        with self._cv:
            self._declare_failed(worker_ids, reason)
            self._cv.notify_all()

    def _declare_failed(self, worker_ids, reason: str) -> None:
        newly = self.membership.mark(worker_ids, WorkerState.FAILED)
        if not newly or self.phase == "finished":
            return
        log.warning("failed: %s (%s)", newly, reason)
        self.history.append(dict(t=time.monotonic(), event="failure", workers=newly, reason=reason))
        for wid in newly:  # fence: its agent SIGKILLs it
            link = self._agents.get(self.membership.workers[wid].node_id)
            if link is not None:
                link.send(P.msg(P.KILL, worker_id=wid, reason=reason))
        self._failures.update(newly)
        self._failed_since_commit += newly

    def _finish_job(self) -> None:
        self.phase = "finished"
        self.history.append(dict(t=time.monotonic(), event="finished", generation=self.committed_generation))
        self._persist()
        self._broadcast(self.membership.alive_ids(), P.msg(P.SHUTDOWN, gen=self.committed_generation))
        log.warning("job finished at generation %d", self.committed_generation)

    def request_replan(self, reason: str) -> None:
        with self._cv:
            self._replan_reason = reason
            self._cv.notify_all()

    def set_health(self, worker_id: str, **health) -> None:
        with self._cv:
            rec = self.membership.workers.get(worker_id)
            if rec is not None:
                rec.health.update(health)

    # ------------------------------------------------------------------ monitor thread
    def _watch(self) -> None:
        while not self._stopped.is_set():
            now = time.monotonic()
            with self._cv:
                self._expire_leases(now)
                if self.phase == "running":
                    self._check_hang(now)
                elif self.phase == "waiting" and self.committed_generation == 0 and not self._start_requested:
                    self._start_requested = self._ready_to_start(now)
                self._cv.notify_all()
            time.sleep(self.tick)

    def _expire_leases(self, now: float) -> None:
        for node in [n for n, seen in self._node_seen.items() if now - seen > self.lease_timeout]:
            del self._node_seen[node]
            victims = [w.worker_id for w in self.membership.on_node(node) if w.alive]
            if victims:
                self._declare_failed(victims, f"node {node} lease expired")

    def _ready_to_start(self, now: float) -> bool:
        count = len(self.membership.alive())
        if self.expected_workers is not None:
            return count >= self.expected_workers
        if self._first_register is None:
            return False
        return count >= self.min_workers and now - self._first_register >= self.start_grace

    def _check_hang(self, now: float) -> None:
        members = [w for w in self.membership.alive() if w.worker_id in self.world]
        if not members or min(now - w.progress_changed_at for w in members) <= self.hang_timeout:
            return
        outside = [w for w in members if not w.progress.get("in_collective", False)]
        if 0 < len(outside) < len(members):
            culprits = outside
        else:  # everyone (or nobody) is inside a collective: blame whoever is furthest behind
            where = {w.worker_id: (w.progress.get("iteration", -1), w.progress.get("op_seq", -1)) for w in members}
            behind = min(where.values())
            culprits = [w for w in members if where[w.worker_id] == behind]
        if len(culprits) < len(members):
            self._declare_failed([w.worker_id for w in culprits], "hang (no progress while peers wait)")
            return
        for w in members:
            w.progress_changed_at = now
        log.error("global stall without an identifiable culprit; extending the deadline")

    # ------------------------------------------------------------------ transaction thread
    def _work_pending(self) -> bool:
        if self._failures or self._start_requested:
            return True
        return bool(self._replan_reason) and self.committed_generation > 0

    def _drive(self) -> None:
        while not self._stopped.is_set():
            with self._cv:
                while not (self._stopped.is_set() or self._work_pending()):
                    self._cv.wait(self.tick)
                if self._stopped.is_set() or self.phase == "finished":
                    return
                failing = bool(self._failures)
                first = self.committed_generation == 0
                reason = "failure" if failing else ("start" if first else (self._replan_reason or "replan"))
                immediate = failing or first or self._force_immediate
                self._replan_reason, self._force_immediate, self._start_requested = None, False, False
            try:
                self._transaction(reason, immediate)
            except Exception:  # noqa: BLE001 -- the authority must not die silently
                log.exception("transaction raised; retrying")
                time.sleep(self.tick)

    def _await(self, condition: Callable[[], bool], timeout: float) -> bool:
        """Wait for ``condition``; raise ``TransactionRestart`` as soon as a failure is declared."""
        deadline = time.monotonic() + timeout
        with self._cv:
            while not condition():
                if self._failures:
                    raise TransactionRestart()
                remaining = deadline - time.monotonic()
                if remaining <= 0 or self._stopped.is_set():
                    return False
                self._cv.wait(min(self.tick, remaining))
        return True

    def _transaction(self, reason: str, immediate: bool) -> None:
        while not self._stopped.is_set():
            with self._cv:
                self._failures.clear()
                self._done.clear()
                self.generation += 1
                self.phase = "reconfiguring"
                attempt = _Attempt(self, self.generation, reason, immediate, self.membership.alive_ids())
                if not self._persist():
                    return
            try:
                attempt.run()
                return  # committed, or leadership lost / stopped
            except TransactionRestart:
                with self._cv:
                    self._open_notice = None
                reason, immediate = "failure", True

    # ------------------------------------------------------------------ introspection
    def wait_for_commit(self, generation: int, timeout: float = 30.0) -> bool:
        deadline = time.monotonic() + timeout
        with self._cv:
            while self.committed_generation < generation:
                remaining = deadline - time.monotonic()
                if remaining <= 0:
                    return False
                self._cv.wait(min(0.05, remaining))
        return True


class _Attempt:
    """One generation's transaction: notice -> plan -> prepare -> commit."""

    def __init__(self, coord: Coordinator, gen: int, reason: str, immediate: bool, participants: list[str]):
        self.c, self.gen, self.reason, self.immediate, self.participants = coord, gen, reason, immediate, participants

    def _event(self, name: str) -> None:
        self.c.history.append(dict(t=time.monotonic(), event=name, generation=self.gen))

    def run(self) -> bool:
        if not self.notice():
            raise TransactionRestart()
        planned = self.plan()
        if planned is None:
            return False
        world, payload, recovery = planned
        self.prepare(world, payload, recovery)
        return self.commit(world, payload)

    def notice(self) -> bool:
        """Announce the generation and collect ABORTED acks (skipped for the very first world)."""
        c = self.c
        if self.reason == "failover":  # let every agent find the new leader first
            c._await(lambda: {w.node_id for w in c.membership.alive()} <= set(c._agents), 2 * c.lease_timeout)
        if not c._prepared_any:
            return True
        note = P.msg(P.RECONFIG_NOTICE, gen=self.gen, failed=list(c._failed_since_commit), immediate=self.immediate,
                     reason=self.reason)
        with c._cv:
            c._open_notice = note
            self._event("notice")
        c._broadcast(self.participants, note)
        acked = c._ledger.aborted[self.gen]
        if c._await(lambda: set(c.membership.alive_ids()) <= set(acked), c.abort_timeout):
            return True
        with c._cv:
            c._open_notice = None
            silent = sorted(set(c.membership.alive_ids()) - set(acked))
            c._declare_failed(silent, "no ABORTED ack within timeout")
        return False

    def plan(self):
        c = self.c
        with c._cv:
            c._open_notice = None
            self._event("aborted")
            recovery = dict(c._ledger.aborted[self.gen])
            alive = [w for w in c.membership.alive() if not c._prepared_any or w.worker_id in recovery]
            c._joiners.difference_update(w.worker_id for w in alive)
            if not c._joiners and (c._replan_reason or "").startswith("join:"):
                c._replan_reason = None
            view = ClusterView(generation=self.gen, alive=alive, failed=list(c._failed_since_commit),
                               previous_world=list(c.world), previous_payload=c.payload, recovery=recovery,
                               reason=self.reason, reports={k: list(v) for k, v in c._reports.items()})
        world, payload = c.planner(view)
        if not world:
            raise RuntimeError("planner returned an empty world")
        with c._cv:
            self._event("planned")
            stored = c._persist() and c._lead.write(f"{c.ns}/plan/{self.gen}",
                                                    json.dumps({"world": world, "payload": payload}))
            if not stored:
                return None
            c._prepared_any = True
        return world, payload, recovery

    def prepare(self, world: list[str], payload: dict, recovery: dict) -> None:
        c = self.c
        with c._cv:
            targets = c.membership.alive_ids()
        c._broadcast(targets, P.msg(P.PREPARE, gen=self.gen, world=world, payload=payload, reason=self.reason,
                                    store_addr=list(c.store_addr) if c.store_addr else None,
                                    store_prefix=f"{c.ns}/gen{self.gen}/", recovery=recovery))
        ready = c._ledger.ready[self.gen]
        if c._await(lambda: set(world) <= ready, c.ready_timeout):
            return
        with c._cv:
            missing = set(world) - ready
            # ranks that reported a failed build were blocked by a peer: blame the silent ones
            blame = (missing - c._ledger.build_failed[self.gen]) or missing
            c._declare_failed(sorted(blame), "no READY within timeout")
        raise TransactionRestart()

    def commit(self, world: list[str], payload: dict) -> bool:
        c = self.c
        with c._cv:
            if c._stopped.is_set():
                return False
            self._event("ready")
            c.committed_generation, c.world, c.payload, c.phase = self.gen, list(world), payload, "running"
            c._failed_since_commit = []
            c._reports.clear()
            now = time.monotonic()
            for w in c.membership.alive():
                w.progress_changed_at = now
            if not c._persist():
                return False
            c.history.append(dict(t=now, event="commit", generation=self.gen, world=list(world), reason=self.reason))
            targets = c.membership.alive_ids()
        c._broadcast(targets, P.msg(P.COMMIT, gen=self.gen))
        log.warning("committed generation %d (%d workers, %s)", self.gen, len(world), self.reason)
        return True
