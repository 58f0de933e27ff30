"""Trace-driven simulation of one long pre-training job under resilience policies.

The job is ``D`` replicas x ``S`` pipeline stages of ``TP``-GPU groups (TP innermost, then
replica, then stage).  Progress is counted in *healthy seconds* -- wall time the failure-free
job would need for the same work -- so ETTR = progress / wall time.  For each event a policy
decides the outage (detection + reconfiguration or restart), the work rolled back, and the
throughput of the degraded cluster until the hardware returns:

* group capacity ``c`` in [0, 1]: a group with lost members shrinks TP (the best feasible degree
  over its survivors, not below ``min_tp``) or is evicted; a detected slow member caps it;
* policies that keep the global batch move *whole* micro-batches: a stage runs at
  ``C_s = M / T_s`` with ``T_s`` the smallest time in which its groups finish ``M``
  micro-batches (``integer_capacity``); without layer repartition the job runs at
  ``min_s C_s / D``, with a perfect one at ``sum_s C_s / (S D)``; ResiHP realises a blend
  ``beta`` of the two, scaled by an ``overhead`` factor, both fitted to the real planner
  (``sim.calibrate``);
* replica-granular policies drop whole replicas (torchft lets the batch shrink, torchft-bp
  keeps it); restart-based ones (NVRx, Greyhound) re-form as many complete replicas as healthy
  plus spare nodes allow; Oobleck runs on whole usable nodes;
* an undetected slowdown stalls the synchronous job by its factor.

(Reference: ``resihp/sim/cluster.py:35-395``; the policy parameters are modelling assumptions
kept identical so results compare.)
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
    """Upper bound: no downtime or rollback, throughput = surviving GPU fraction."""
    return PolicyParams("Ideal", detect_s=0.0, reconfig_s=0.0, lost_iterations=0.0, job_restart_s=0.0,
                        job_rollback_s=0.0, ideal=True)


def resihp_params(job: JobConfig, *, comm_rebuild_s: float = 10.0, migrate_s: float = 5.0, snapshot_iters: int = 10,
                  beta: float = 0.5, overhead: float = 1.0, slow_detect_iters: float = 3.0) -> PolicyParams:
    return PolicyParams("ResiHP", detect_s=3.0, reconfig_s=comm_rebuild_s + migrate_s + job.iteration_s,
                        lost_iterations=0.5, job_restart_s=120.0, job_rollback_s=snapshot_iters / 2 * job.iteration_s,
                        repair_s=comm_rebuild_s + migrate_s, tp_shrink=True, migrate=True, beta=beta, overhead=overhead,
                        slow_detect_s=slow_detect_iters * job.iteration_s, slow_mitigation="migrate")


def baseline_params(job: JobConfig, *, restart_s: float = 300.0,
                    checkpoint_interval_s: float = 1200.0) -> list[PolicyParams]:
    ck = dict(checkpoint_interval_s=checkpoint_interval_s)
    return [
        PolicyParams("torchft", detect_s=10.0, reconfig_s=15.0, job_restart_s=restart_s, repair_s=15.0,
                     replica_granular=True, keep_batch=False, **ck),
        PolicyParams("torchft-bp", detect_s=10.0, reconfig_s=15.0, job_restart_s=restart_s, repair_s=15.0,
                     replica_granular=True, **ck),
        PolicyParams("NVRx", detect_s=60.0, reconfig_s=0.0, restart_s=restart_s, job_restart_s=restart_s,
                     restart_on_fail=True, replica_granular=True, slow_detect_s=300.0,
                     slow_mitigation="exclude_node", **ck),
        PolicyParams("ReCycle", detect_s=10.0, reconfig_s=15.0, job_restart_s=restart_s, repair_s=15.0, migrate=True,
                     **ck),
        PolicyParams("Oobleck", detect_s=10.0, reconfig_s=60.0, job_restart_s=restart_s, repair_s=60.0,
                     node_granular=True, **ck),
        PolicyParams("Greyhound", detect_s=60.0, reconfig_s=0.0, restart_s=restart_s, job_restart_s=restart_s,
                     restart_on_fail=True, replica_granular=True, migrate=True, slow_detect_s=10 * job.iteration_s,
                     slow_mitigation="migrate", **ck),
    ]


def integer_capacity(caps: list[float], microbatches: int) -> float:
    """Throughput (in healthy-group units) of groups with relative speeds ``caps`` that split
    ``microbatches`` whole micro-batches optimally: ``M / T*`` with ``T*`` the smallest time
    such that ``sum_r floor(T* c_r) >= M``.  Exact: start from the fluid bound ``M / sum c``
    and advance to the next completion instant of the group that finishes soonest until ``M``
    micro-batches are done (at most one step per group)."""
    live = [c for c in caps if c > 0]
    if not live:
        return 0.0
    M = microbatches
    t = M / sum(live)
    done = [math.floor(t * c + 1e-9) for c in live]
    total = sum(done)
    if total >= M:
        return M / t
    heap = [((done[i] + 1) / c, i) for i, c in enumerate(live)]
    heapq.heapify(heap)
    while total < M:
        t, i = heapq.heappop(heap)
        done[i] += 1
        total += 1
        heapq.heappush(heap, ((done[i] + 1) / live[i], i))
    return M / t


class ClusterState:
    """Hardware state as one policy sees it: lost GPUs (until repaired), spare nodes in use,
    slow GPUs and the capacity of every (replica, stage) group."""

    def __init__(self, job: JobConfig, p: PolicyParams):
        self.job, self.p = job, p
        self.lost: dict[int, float] = {}            # GPU -> repair time (degrading capacity)
        self.failed: dict[int, float] = {}          # GPU -> repair time (incl. spare-covered)
        self.slow: dict[int, tuple[float, float, bool]] = {}  # GPU -> (factor, until, detected)
        self.covered: set[int] = set()              # failed nodes replaced by a spare
        self.spares_free = job.spare_nodes
        self.spares = 0
        self.c = [[1.0] * job.pp for _ in range(job.dp)]
        self.stage_cap = [float(job.dp)] * job.pp

    # -- hardware events
    def fail(self, gpus, until: float) -> tuple[list[int], int]:
        """Returns the GPUs that now reduce capacity and the number of spare nodes used."""
        gpn = self.job.gpus_per_node
        for g in gpus:
            self.failed[g] = max(self.failed.get(g, 0.0), until)
        used, degrading = 0, []
        for node in sorted({g // gpn for g in gpus}):
            if node in self.covered:
                continue
            if self.spares_free > 0:
                self.spares_free -= 1
                self.covered.add(node)
                used += 1
                for g in range(node * gpn, (node + 1) * gpn):
                    self.lost.pop(g, None)
            else:
                degrading += [g for g in gpus if g // gpn == node and g not in self.lost]
        for g in degrading:
            self.lost[g] = self.failed[g]
        return degrading, used

    def repair(self, gpus, now: float) -> list[int]:
        gpn = self.job.gpus_per_node
        back = [g for g in gpus if g in self.failed and self.failed[g] <= now + 1e-6]
        for g in back:
            del self.failed[g]
            self.lost.pop(g, None)
        for node in {g // gpn for g in back}:
            if node in self.covered and not any(h // gpn == node for h in self.failed):
                self.covered.discard(node)
                self.spares_free += 1
        return back

    # -- capacities
    def _known_speed(self, g: int) -> float:
        f = self.slow.get(g)
        return 1.0 / f[0] if f is not None and f[2] else 1.0  # undetected: invisible to the planner

    def _group_capacity(self, r: int, s: int) -> float:
        job, p = self.job, self.p
        speeds = sorted((self._known_speed(g) for g in job.group_gpus(r, s) if g not in self.lost), reverse=True)
        if not speeds or (len(speeds) < job.tp and not p.tp_shrink):
            return 0.0
        full = job.profile.group_speed(job.tp, 1.0)
        if not p.tp_shrink:
            return job.profile.group_speed(job.tp, speeds[-1]) / full
        # Eq. 4 over the survivors: the k fastest at the slowest of them
        return max((job.profile.group_speed(k, speeds[k - 1]) / full
                    for k in job.tp_degrees if job.min_tp <= k <= len(speeds)), default=0.0)

    def refresh(self, gpus) -> None:
        for r, s in {self.job.group_of(g) for g in gpus}:
            self.c[r][s] = self._group_capacity(r, s)
            self.stage_cap[s] = integer_capacity([self.c[x][s] for x in range(self.job.dp)], self.job.microbatches)

    # -- throughput (fraction of healthy)
    def throughput(self) -> float:
        job, p = self.job, self.p
        if p.ideal:
            return (job.gpus - len(self.lost)) / job.gpus
        hidden = [f for f, _, detected in self.slow.values() if not detected]
        sync = 1.0 / max(hidden) if hidden else 1.0
        if p.node_granular:
            return self._node_granular() * sync
        if p.replica_granular:
            return self._replica_granular() * sync
        if not p.migrate:
            return min(min(row) for row in self.c) * sync
        D, S = job.dp, job.pp
        bottleneck = min(self.stage_cap) / D
        spread = sum(self.stage_cap) / (S * D)
        blend = (1 - p.beta) * bottleneck + p.beta * spread
        return max(0.0, 1.0 - p.overhead * (1.0 - blend)) * sync

    def _node_granular(self) -> float:
        job = self.job
        bad = {g // job.gpus_per_node for g in self.lost}
        if not bad:
            return 1.0
        usable = max(0, job.nodes - max(0, len(bad) - self.spares))
        return 0.95 * usable / job.nodes

    def _replica_granular(self) -> float:
        job, p = self.job, self.p
        D = job.dp
        bad = set(self.lost)
        if p.slow_mitigation == "exclude_node":
            bad |= {g for g, (_, _, detected) in self.slow.items() if detected}
        if p.restart_on_fail:
            bad_nodes = {g // job.gpus_per_node for g in bad}
            up = min(D, (job.nodes - len(bad_nodes) + self.spares) // job.nodes_per_replica())
        else:
            down = {job.group_of(g)[0] for g in bad}
            up = D - max(0, len(down) - self.spares)
        if up <= 0:
            return 0.0
        caps = [1.0] * up
        if p.slow_mitigation == "migrate":
            for g, (f, _, detected) in self.slow.items():
                r = job.group_of(g)[0]
                if detected and r < up:
                    caps[r] = min(caps[r], 1.0 / f)
        if not p.keep_batch:
            return sum(caps) / D
        return integer_capacity(caps, job.microbatches) / D


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
        n = len(self.mttr_s)
        srt = sorted(self.mttr_s)
        return {"policy": self.policy, "gpus": self.gpus, "ettr": self.ettr,
                "downtime_frac": self.downtime_s / self.horizon_s, "lost_frac": self.lost_s / self.horizon_s,
                "degraded_frac": self.degraded_loss_s / self.horizon_s, "events": self.events,
                "mttr_mean_s": sum(srt) / n if n else 0.0, "mttr_p99_s": srt[int(0.99 * (n - 1))] if n else 0.0}


class _Run:
    """Accounting of one simulation: progress integrates throughput outside outages; outages
    charge downtime and roll progress back; checkpoints mark the rollback target."""

    def __init__(self, st: ClusterState, p: PolicyParams):
        self.st, self.p = st, p
        self.t = self.progress = self.downtime = self.lost = self.degraded = 0.0
        self.busy_until = 0.0
        self.ckpt_progress = 0.0
        self.next_ckpt = p.checkpoint_interval_s
        self.mttr: list[float] = []

    def advance(self, to: float) -> None:
        while self.t < to:
            seg_end = min(to, self.next_ckpt)
            start = max(self.t, self.busy_until)
            if seg_end > start:
                thr = self.st.throughput()
                self.progress += thr * (seg_end - start)
                self.degraded += (1.0 - thr) * (seg_end - start)
            self.t = seg_end
            if self.t >= self.next_ckpt:
                self.ckpt_progress = self.progress
                self.next_ckpt += self.p.checkpoint_interval_s

    def outage(self, cost: float, rollback: float) -> None:
        start = max(self.t, self.busy_until)
        self.busy_until = start + cost
        self.downtime += cost
        rb = min(rollback, self.progress)
        self.progress -= rb
        self.lost += rb
        self.mttr.append(cost)

    def since_checkpoint(self) -> float:
        return self.progress - self.ckpt_progress


def simulate(events: list[Event], job: JobConfig, p: PolicyParams, horizon_s: float) -> SimResult:
    st = ClusterState(job, p)
    run = _Run(st, p)
    heap: list[tuple[float, int, str, object]] = []
    seq = 0

    def push(when: float, kind: str, obj) -> None:
        nonlocal seq
        heapq.heappush(heap, (when, seq, kind, obj))
        seq += 1

    for e in events:
        if e.t < horizon_s:
            push(e.t, "event", e)
    while heap:
        when, _, kind, obj = heapq.heappop(heap)
        if when >= horizon_s:
            break
        run.advance(when)
        if kind == "event":
            e: Event = obj
            if e.kind == "fail" and e.domain == "job":
                rb = p.job_rollback_s if p.job_rollback_s is not None else run.since_checkpoint()
                run.outage(p.detect_s + p.job_restart_s, rb)
            elif e.kind == "fail":
                _, spares_used = st.fail(e.targets, when + e.duration_s)
                st.refresh(e.targets)
                if p.restart_on_fail:
                    run.outage(p.detect_s + p.restart_s, run.since_checkpoint())
                else:  # integrating a spare costs one more planned reconfiguration
                    extra = p.repair_s if spares_used else 0.0
                    run.outage(p.detect_s + p.reconfig_s + extra, p.lost_iterations * job.iteration_s)
                push(when + e.duration_s, "repair", tuple(e.targets))
            elif e.kind == "slow":
                g = e.targets[0]
                st.slow[g] = (e.factor, when + e.duration_s, False)
                st.refresh([g])
                if p.slow_detect_s is not None and p.slow_detect_s < e.duration_s:
                    push(when + p.slow_detect_s, "slow_detected", g)
                push(when + e.duration_s, "slow_end", g)
            elif e.kind == "planned":
                run.outage(p.job_restart_s if p.restart_on_fail else p.reconfig_s, 0.0)
        elif kind == "repair":
            was_degraded = any(g in st.lost for g in obj)
            back = st.repair(obj, when)
            if back:
                st.refresh(back)
                if was_degraded and p.repair_s and not p.restart_on_fail:
                    run.outage(p.repair_s, 0.0)
        elif kind == "slow_detected":
            g = obj
            if g in st.slow:
                f, until, _ = st.slow[g]
                st.slow[g] = (f, until, True)
                st.refresh([g])
                if p.slow_mitigation == "exclude_node":
                    run.outage(p.detect_s + p.restart_s, run.since_checkpoint())
                elif p.slow_mitigation == "migrate":
                    run.outage(0.0 if p.restart_on_fail else p.reconfig_s, 0.0)
        elif kind == "slow_end":
            if obj in st.slow:
                del st.slow[obj]
                st.refresh([obj])
    run.advance(horizon_s)
    return SimResult(p.name, job.gpus, horizon_s, run.progress, run.downtime, run.lost, run.degraded,
                     len(run.mttr), run.mttr)
