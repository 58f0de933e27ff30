"""Trace-driven simulation of one long pre-training job under a resilience policy.

The job is ``D`` replicas x ``S`` pipeline stages of ``TP``-GPU groups (TP innermost, then
replica, then stage).  Progress is counted in *healthy seconds* -- the wall time the
failure-free job would need for the same work -- so ETTR = progress / wall time.  For every
event the policy decides the outage (detection plus reconfiguration, or a restart), the work
rolled back, and the throughput of the degraded cluster until the hardware returns:

* a group's capacity ``c`` in [0, 1]: a group that lost members shrinks TP (the best feasible
  degree over its survivors, not below ``min_tp``) or is evicted; a detected slow member caps it;
* a policy that keeps the global batch moves *whole* micro-batches: stage ``s`` runs at
  ``C_s = M / T_s`` with ``T_s`` the least time in which its groups finish ``M`` micro-batches
  (``integer_capacity``).  Without layer repartition the job runs at ``min_s C_s / D``, with a
  perfect one at ``sum_s C_s / (S D)``; ResiHP realises a blend ``beta`` of the two, scaled by
  an ``overhead`` factor -- both fitted to the real planner (``sim.calibrate``);
* replica-granular policies drop whole replicas (torchft lets the batch shrink, torchft-bp keeps
  it); restart-based ones (NVRx, Greyhound) re-form as many complete replicas as the healthy and
  spare nodes allow; Oobleck runs on whole usable nodes;
* an undetected slowdown stalls the synchronous job by its factor.

Parity: ``resihp/sim/cluster.py:35-395``.  The policy parameters are modelling assumptions and
are kept identical so results compare; the simulation code is ours (exact integer capacity by
completion-instant stepping, hardware state and capacity model split, an event-handler table).
"""

from __future__ import annotations

import heapq
import math
from dataclasses import dataclass, field

from ..plan.model_spec import ModelProfile
from .traces import Event


@dataclass
class JobConfig:
    gpus: int
    tp: int = 8
    pp: int = 16
    gpus_per_node: int = 8
    iteration_s: float = 12.0
    microbatches_per_replica: int = 16
    min_tp: int = 4
    tp_degrees: tuple[int, ...] = (1, 2, 4, 8)   # degrees the head / KV-group / FFN sizes divide into
    spare_nodes: int = 0
    profile: ModelProfile = field(default_factory=lambda: ModelProfile(alpha=1.0, beta=0.0))

    @property
    def dp(self) -> int:
        return self.gpus // (self.tp * self.pp)

    @property
    def nodes(self) -> int:
        return self.gpus // self.gpus_per_node

    @property
    def microbatches(self) -> int:
        return self.microbatches_per_replica * self.dp

    def group_of(self, gpu: int) -> tuple[int, int]:
        """(replica, stage) of a GPU."""
        return (gpu // self.tp) % self.dp, gpu // (self.tp * self.dp)

    def group_gpus(self, replica: int, stage: int) -> range:
        base = (stage * self.dp + replica) * self.tp
        return range(base, base + self.tp)

    def nodes_per_replica(self) -> int:
        return self.tp * self.pp // self.gpus_per_node


@dataclass
class PolicyParams:
    name: str
    detect_s: float
    reconfig_s: float
    lost_iterations: float = 0.5        # work lost by an online reconfiguration, in iterations
    restart_s: float = 0.0              # restart of the job after a failure (restart-based policies)
    checkpoint_interval_s: float = 1800.0
    job_restart_s: float = 600.0        # full restart after a job-domain failure
    job_rollback_s: float | None = None  # None: back to the last checkpoint
    repair_s: float = 0.0               # reconfiguration to take returning hardware back
    tp_shrink: bool = False
    migrate: bool = False
    beta: float = 0.0
    overhead: float = 1.0
    slow_detect_s: float | None = None
    slow_mitigation: str = "none"       # none | migrate | exclude_node
    node_granular: bool = False
    replica_granular: bool = False
    restart_on_fail: bool = False
    keep_batch: bool = True
    ideal: bool = False


def ideal_params() -> PolicyParams:
    """Upper bound: no downtime or rollback; throughput = the surviving GPU fraction."""
    return PolicyParams("Ideal", detect_s=0.0, reconfig_s=0.0, lost_iterations=0.0, job_restart_s=0.0,
                        job_rollback_s=0.0, ideal=True)


def resihp_params(job: JobConfig, *, comm_rebuild_s: float = 10.0, migrate_s: float = 5.0, snapshot_iters: int = 10,
                  beta: float = 0.5, overhead: float = 1.0, slow_detect_iters: float = 3.0) -> PolicyParams:
    rebuild = comm_rebuild_s + migrate_s
    return PolicyParams("ResiHP", detect_s=3.0, reconfig_s=rebuild + job.iteration_s, lost_iterations=0.5,
                        job_restart_s=120.0, job_rollback_s=0.5 * snapshot_iters * job.iteration_s, repair_s=rebuild,
                        tp_shrink=True, migrate=True, beta=beta, overhead=overhead,
                        slow_detect_s=slow_detect_iters * job.iteration_s, slow_mitigation="migrate")


def baseline_params(job: JobConfig, *, restart_s: float = 300.0,
                    checkpoint_interval_s: float = 1200.0) -> list[PolicyParams]:
    """torchft, torchft-bp, NVRx, ReCycle, Oobleck and Greyhound as modelled policies."""
    common = dict(checkpoint_interval_s=checkpoint_interval_s, job_restart_s=restart_s)
    online = dict(detect_s=10.0, reconfig_s=15.0, repair_s=15.0, **common)
    restarting = dict(detect_s=60.0, reconfig_s=0.0, restart_s=restart_s, restart_on_fail=True,
                      replica_granular=True, **common)
    return [
        PolicyParams("torchft", replica_granular=True, keep_batch=False, **online),
        PolicyParams("torchft-bp", replica_granular=True, **online),
        PolicyParams("NVRx", slow_detect_s=300.0, slow_mitigation="exclude_node", **restarting),
        PolicyParams("ReCycle", migrate=True, **online),
        PolicyParams("Oobleck", node_granular=True, **dict(online, reconfig_s=60.0, repair_s=60.0)),
        PolicyParams("Greyhound", migrate=True, slow_detect_s=10 * job.iteration_s, slow_mitigation="migrate",
                     **restarting),
    ]


def integer_capacity(caps: list[float], microbatches: int) -> float:
    """Throughput (in healthy-group units) of groups with relative speeds ``caps`` that share
    ``microbatches`` whole micro-batches optimally: ``M / T*`` with ``T*`` the least time such
    that ``sum_r floor(T* c_r) >= M``.  Exact: start at the fluid bound ``M / sum c`` and step to
    the next completion instant of whichever group finishes soonest until ``M`` are done (at most
    one step per group)."""
    speeds = [c for c in caps if c > 0]
    if not speeds:
        return 0.0
    t = microbatches / sum(speeds)
    finished = [math.floor(t * c + 1e-9) for c in speeds]
    if sum(finished) >= microbatches:
        return microbatches / t
    upcoming = [((n + 1) / c, i) for i, (n, c) in enumerate(zip(finished, speeds))]
    heapq.heapify(upcoming)
    for _ in range(microbatches - sum(finished)):
        t, i = heapq.heappop(upcoming)
        finished[i] += 1
        heapq.heappush(upcoming, ((finished[i] + 1) / speeds[i], i))
    return microbatches / t


class ClusterState:
    """The hardware as one policy sees it -- lost GPUs (until repaired), spare nodes in use,
    slow GPUs -- and the capacity of every (replica, stage) group."""

    def __init__(self, job: JobConfig, p: PolicyParams):
        self.job, self.p = job, p
        self.lost: dict[int, float] = {}            # GPU -> repair time; these reduce capacity
        self.failed: dict[int, float] = {}          # GPU -> repair time, spare-covered ones included
        self.slow: dict[int, tuple[float, float, bool]] = {}  # GPU -> (factor, until, detected)
        self.covered: set[int] = set()              # failed nodes a spare node stands in for
        self.spares_free = job.spare_nodes
        self.spares = 0
        self.c = [[1.0] * job.pp for _ in range(job.dp)]
        self.stage_cap = [float(job.dp)] * job.pp

    def _node(self, gpu: int) -> int:
        return gpu // self.job.gpus_per_node

    def _node_gpus(self, node: int) -> range:
        per = self.job.gpus_per_node
        return range(node * per, (node + 1) * per)

    # ---------------------------------------------------------------- hardware events
    def fail(self, gpus, until: float) -> tuple[list[int], int]:
        """Record failed GPUs; a spare node (if free) covers each failed node.  Returns the GPUs
        that now reduce capacity and the number of spare nodes taken."""
        for g in gpus:
            self.failed[g] = max(until, self.failed.get(g, 0.0))
        taken, degrading = 0, []
        for node in sorted(set(map(self._node, gpus)) - self.covered):
            if self.spares_free > 0:
                self.spares_free -= 1
                taken += 1
                self.covered.add(node)
                for g in self._node_gpus(node):
                    self.lost.pop(g, None)
            else:
                degrading += [g for g in gpus if self._node(g) == node and g not in self.lost]
        self.lost.update((g, self.failed[g]) for g in degrading)
        return degrading, taken

    def repair(self, gpus, now: float) -> list[int]:
        back = [g for g in gpus if g in self.failed and self.failed[g] <= now + 1e-6]
        for g in back:
            self.failed.pop(g)
            self.lost.pop(g, None)
        still_failed = set(map(self._node, self.failed))
        for node in set(map(self._node, back)) & self.covered:
            if node not in still_failed:
                self.covered.discard(node)
                self.spares_free += 1
        return back

    # ---------------------------------------------------------------- capacities
    def _visible_speed(self, g: int) -> float:
        """A slow GPU counts as slow only once detected (until then the planner cannot see it)."""
        factor, _until, detected = self.slow.get(g, (1.0, 0.0, False))
        return 1.0 / factor if detected else 1.0

    def _group_capacity(self, r: int, s: int) -> float:
        job, p = self.job, self.p
        alive = sorted((self._visible_speed(g) for g in job.group_gpus(r, s) if g not in self.lost), reverse=True)
        nominal = job.profile.group_speed(job.tp, 1.0)
        if not alive or (not p.tp_shrink and len(alive) < job.tp):
            return 0.0
        if not p.tp_shrink:
            return job.profile.group_speed(job.tp, alive[-1]) / nominal
        # Eq. 4 over the survivors: the k fastest, paced by the slowest of them
        options = [job.profile.group_speed(k, alive[k - 1]) / nominal
                   for k in job.tp_degrees if job.min_tp <= k <= len(alive)]
        return max(options, default=0.0)

    def refresh(self, gpus) -> None:
        for r, s in {self.job.group_of(g) for g in gpus}:
            self.c[r][s] = self._group_capacity(r, s)
            self.stage_cap[s] = integer_capacity([row[s] for row in self.c], self.job.microbatches)

    # ---------------------------------------------------------------- throughput (fraction of healthy)
    def throughput(self) -> float:
        job, p = self.job, self.p
        if p.ideal:
            return (job.gpus - len(self.lost)) / job.gpus
        hidden = [factor for factor, _, detected in self.slow.values() if not detected]
        stall = 1.0 / max(hidden) if hidden else 1.0
        if p.node_granular:
            return stall * self._node_granular()
        if p.replica_granular:
            return stall * self._replica_granular()
        if not p.migrate:
            return stall * min(map(min, self.c))
        bottleneck = min(self.stage_cap) / job.dp
        spread = sum(self.stage_cap) / (job.pp * job.dp)
        blended = p.beta * spread + (1.0 - p.beta) * bottleneck
        return stall * max(0.0, 1.0 - p.overhead * (1.0 - blended))

    def _node_granular(self) -> float:
        bad_nodes = set(map(self._node, self.lost))
        if not bad_nodes:
            return 1.0
        usable = max(0, self.job.nodes - max(0, len(bad_nodes) - self.spares))
        return 0.95 * usable / self.job.nodes

    def _replica_granular(self) -> float:
        job, p = self.job, self.p
        bad = set(self.lost)
        if p.slow_mitigation == "exclude_node":
            bad.update(g for g, (_, _, detected) in self.slow.items() if detected)
        if p.restart_on_fail:
            healthy_nodes = job.nodes - len(set(map(self._node, bad))) + self.spares
            replicas = min(job.dp, healthy_nodes // job.nodes_per_replica())
        else:
            replicas = job.dp - max(0, len({job.group_of(g)[0] for g in bad}) - self.spares)
        if replicas <= 0:
            return 0.0
        caps = [1.0] * replicas
        if p.slow_mitigation == "migrate":
            for g, (factor, _, detected) in self.slow.items():
                r = job.group_of(g)[0]
                if detected and r < replicas:
                    caps[r] = min(caps[r], 1.0 / factor)
        if p.keep_batch:
            return integer_capacity(caps, job.microbatches) / job.dp
        return sum(caps) / job.dp


@dataclass
class SimResult:
    policy: str
    gpus: int
    horizon_s: float
    progress_s: float
    downtime_s: float
    lost_s: float
    degraded_loss_s: float
    events: int
    mttr_s: list[float]

    @property
    def ettr(self) -> float:
        return self.progress_s / self.horizon_s

    def to_json(self) -> dict:
        outages = sorted(self.mttr_s)
        n = len(outages)
        return {"policy": self.policy, "gpus": self.gpus, "ettr": self.ettr,
                "downtime_frac": self.downtime_s / self.horizon_s, "lost_frac": self.lost_s / self.horizon_s,
                "degraded_frac": self.degraded_loss_s / self.horizon_s, "events": self.events,
                "mttr_mean_s": sum(outages) / n if n else 0.0, "mttr_p99_s": outages[int(0.99 * (n - 1))] if n else 0.0}


class _Ledger:
    """Progress integrates throughput outside outages; an outage charges downtime and rolls
    progress back; checkpoints mark the rollback target."""

    def __init__(self, st: ClusterState, p: PolicyParams):
        self.st, self.p = st, p
        self.t = self.progress = self.downtime = self.lost = self.degraded = 0.0
        self.blocked_until = 0.0
        self.checkpointed = 0.0
        self.next_checkpoint = p.checkpoint_interval_s
        self.outages: list[float] = []

    def advance(self, until: float) -> None:
        while self.t < until:
            stop = min(until, self.next_checkpoint)
            begin = max(self.t, self.blocked_until)
            if stop > begin:
                rate = self.st.throughput()
                self.progress += rate * (stop - begin)
                self.degraded += (1.0 - rate) * (stop - begin)
            self.t = stop
            if self.t >= self.next_checkpoint:
                self.checkpointed = self.progress
                self.next_checkpoint += self.p.checkpoint_interval_s

    def outage(self, cost: float, rollback: float) -> None:
        self.blocked_until = max(self.t, self.blocked_until) + cost
        self.downtime += cost
        undone = min(rollback, self.progress)
        self.progress -= undone
        self.lost += undone
        self.outages.append(cost)

    def since_checkpoint(self) -> float:
        return self.progress - self.checkpointed


class _Simulation:
    def __init__(self, job: JobConfig, p: PolicyParams, horizon_s: float):
        self.job, self.p, self.horizon = job, p, horizon_s
        self.st = ClusterState(job, p)
        self.ledger = _Ledger(self.st, p)
        self.queue: list[tuple[float, int, str, object]] = []
        self.seq = 0

    def push(self, when: float, kind: str, what) -> None:
        heapq.heappush(self.queue, (when, self.seq, kind, what))
        self.seq += 1

    def run(self, events: list[Event]) -> SimResult:
        for e in events:
            if e.t < self.horizon:
                self.push(e.t, e.kind, e)
        while self.queue:
            when, _, kind, what = heapq.heappop(self.queue)
            if when >= self.horizon:
                break
            self.ledger.advance(when)
            getattr(self, f"_on_{kind}")(when, what)
        self.ledger.advance(self.horizon)
        led = self.ledger
        return SimResult(self.p.name, self.job.gpus, self.horizon, led.progress, led.downtime, led.lost, led.degraded,
                         len(led.outages), led.outages)

    def _on_fail(self, when: float, e: Event) -> None:
        p, led = self.p, self.ledger
        if e.domain == "job":  # everyone restarts; nothing is lost
            rollback = p.job_rollback_s if p.job_rollback_s is not None else led.since_checkpoint()
            led.outage(p.detect_s + p.job_restart_s, rollback)
            return
        _, spares_taken = self.st.fail(e.targets, when + e.duration_s)
        self.st.refresh(e.targets)
        if p.restart_on_fail:
            led.outage(p.detect_s + p.restart_s, led.since_checkpoint())
        else:  # taking a spare in costs one more planned reconfiguration
            extra = p.repair_s if spares_taken else 0.0
            led.outage(p.detect_s + p.reconfig_s + extra, p.lost_iterations * self.job.iteration_s)
        self.push(when + e.duration_s, "repair", tuple(e.targets))

    def _on_slow(self, when: float, e: Event) -> None:
        g = e.targets[0]
        self.st.slow[g] = (e.factor, when + e.duration_s, False)
        self.st.refresh([g])
        if self.p.slow_detect_s is not None and self.p.slow_detect_s < e.duration_s:
            self.push(when + self.p.slow_detect_s, "slow_detected", g)
        self.push(when + e.duration_s, "slow_end", g)

    def _on_planned(self, when: float, e: Event) -> None:
        self.ledger.outage(self.p.job_restart_s if self.p.restart_on_fail else self.p.reconfig_s, 0.0)

    def _on_repair(self, when: float, gpus) -> None:
        was_degraded = any(g in self.st.lost for g in gpus)
        back = self.st.repair(gpus, when)
        if not back:
            return
        self.st.refresh(back)
        if was_degraded and self.p.repair_s and not self.p.restart_on_fail:
            self.ledger.outage(self.p.repair_s, 0.0)

    def _on_slow_detected(self, when: float, g: int) -> None:
        if g not in self.st.slow:
            return
        factor, until, _ = self.st.slow[g]
        self.st.slow[g] = (factor, until, True)
        self.st.refresh([g])
        p = self.p
        if p.slow_mitigation == "exclude_node":
            self.ledger.outage(p.detect_s + p.restart_s, self.ledger.since_checkpoint())
        elif p.slow_mitigation == "migrate":
            self.ledger.outage(0.0 if p.restart_on_fail else p.reconfig_s, 0.0)

    def _on_slow_end(self, when: float, g: int) -> None:
        if self.st.slow.pop(g, None) is not None:
            self.st.refresh([g])


def simulate(events: list[Event], job: JobConfig, p: PolicyParams, horizon_s: float) -> SimResult:
    return _Simulation(job, p, horizon_s).run(events)
