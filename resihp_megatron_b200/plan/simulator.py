"""List-scheduling pipeline simulator, shared by the planner and the fail-slow detector.

Given a plan and cost functions it produces, per physical slot, a concrete compute order
(1F1B-like under an in-flight limit, with optional zero-bubble W ops), the timing of every op,
each slot's peak number of in-flight micro-batches and the makespan.  Messages travel on
physical ``(source slot, destination slot, kind)`` channels consumed strictly in send order --
the discipline that keeps NCCL point-to-point safe -- so every order converts to a valid IR.

Rule: repeatedly run, over all slots, the ready op with the earliest start time.  Ties go to
backward before forward before weight-gradient, then the lower micro-batch, then the lower
stage (within a slot) or the lower slot key (across slots).  A slot's ready ops are: the next
micro-batch's first-stage forward (under the in-flight limit); forwards whose activation sits at
the head of an incoming channel (the limit applies to the slot's first chunk); the oldest
pending last-stage backward; backwards whose gradient heads an incoming channel; queued W ops.
Parity: ``resihp/plan/simulator.py:45-251`` (same rule, limits and interleaved order).
"""

from __future__ import annotations

import math
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Callable

from .hetero_plan import HeteroParallelPlan

Key = tuple[int, int]
CostFn = Callable[[Key, str, int], float]
CommFn = Callable[[Key, Key, str], float]

_RANK = {"B": 0, "F": 1, "W": 2}


@dataclass
class SimOp:
    key: Key
    op: str
    mb: int
    start: float
    end: float
    stage: int | None = None


@dataclass
class SimResult:
    order: dict[Key, list[tuple]]
    ops: list[SimOp]
    makespan: float
    finish: dict[Key, float]
    busy: dict[Key, float]
    peak_inflight: dict[Key, int]
    deadlock: bool = False
    stage_forward_done: dict[Key, float] = field(default_factory=dict)


def default_inflight_limit(plan: HeteroParallelPlan) -> dict[Key, float]:
    """How many micro-batches a physical slot may hold between first forward and last backward.

    Plain 1F1B: the warm-up depth ``P - p`` scaled by the slot's share of its stage's
    micro-batches (a slot that absorbed migrated micro-batches needs proportionally deeper
    warm-up).  Interleaved: only the pipeline entry is limited, to the interleaved warm-up depth;
    that bounds every slot, whereas per-slot limits could stall a chunk-0 message at a channel
    head in front of a chunk-1 message."""
    P, v = plan.num_physical_stages, plan.vpp
    entry_depth = math.ceil(((P - 1) * 2 + (v - 1) * P) / v) + 1
    limits: dict[Key, float] = {}
    for g in plan.stage_groups:
        slot = plan.physical_key(g.replica, g.stage)
        r, p = slot
        if v > 1:
            limits[slot] = entry_depth if p == 0 else math.inf
            continue
        share = len(plan.microbatches_of(r, p)) * plan.num_replicas / plan.num_microbatches
        limits[slot] = max(1, math.ceil((P - p) * max(1.0, share)))
    return limits


def megatron_interleaved_order(plan: HeteroParallelPlan, split_backward: bool = False):
    """Megatron's static interleaved 1F1B order per physical slot: forwards in rounds of ``P``
    micro-batches chunk by chunk, backwards with the chunks reversed, a warm-up of
    ``(P - p - 1) * 2 + (v - 1) * P`` forwards; a split backward puts each W right after its B.
    ``None`` when the chunks of a slot run different micro-batch sets."""
    P, v = plan.num_physical_stages, plan.vpp
    orders: dict[Key, list[tuple]] = {}
    for g in plan.stage_groups:
        slot = plan.physical_key(g.replica, g.stage)
        if slot in orders:
            continue
        r, p = slot
        mbs = plan.microbatches_of(r, p)
        same_set = all(plan.group(r, p + c * P) is not None and plan.microbatches_of(r, p + c * P) == mbs
                       for c in range(v))
        if not same_set:
            return None
        n = len(mbs)
        total = n * v

        def item(k: int, backward: bool) -> tuple[int, int]:
            round_start = (k // (P * v)) * P
            width = min(P, n - round_start)
            chunk, i = divmod(k - round_start * v, width)
            if backward:
                chunk = v - 1 - chunk
            return mbs[round_start + i], chunk * P + p

        warm = min(total, (P - p - 1) * 2 + (v - 1) * P)
        seq = [("F", *item(k, False)) for k in range(warm)]
        backs = []
        for k in range(total):
            mb, s = item(k, True)
            backs.append([("B", mb, s)] + ([("W", mb, s)] if split_backward else []))
        for k in range(total - warm):
            seq.append(("F", *item(warm + k, False)))
            seq.extend(backs[k])
        for k in range(total - warm, total):
            seq.extend(backs[k])
        orders[slot] = seq
    return orders


class _Scheduler:
    def __init__(self, plan, cost, comm, split_backward, inflight_limit, fixed):
        self.plan, self.cost, self.comm, self.split, self.fixed = plan, cost, comm, split_backward, fixed
        self.S, self.interleaved = plan.num_stages, plan.vpp > 1
        units = [(g.replica, g.stage) for g in plan.stage_groups]
        self.slot_of = {u: plan.physical_key(*u) for u in units}
        self.slots = sorted(set(self.slot_of.values()))
        self.chunks = {k: sorted(u[1] for u in units if self.slot_of[u] == k) for k in self.slots}
        self.limit = default_inflight_limit(plan) if inflight_limit is None else inflight_limit
        self.entry_queue = {u: [m for m in range(plan.num_microbatches) if plan.executor(u[1], m) == u[0]]
                            for u in units}
        self.remaining = sum(map(len, self.entry_queue.values())) * (3 if split_backward else 2)
        self.fwd_end = {u: {} for u in units}
        self.bwd_end = {u: {} for u in units}
        self.w_queue = {k: [] for k in self.slots}
        self.clock = dict.fromkeys(self.slots, 0.0)
        self.busy = dict.fromkeys(self.slots, 0.0)
        self.holding = dict.fromkeys(self.slots, 0)
        self.peak = dict.fromkeys(self.slots, 0)
        self.order = {k: [] for k in self.slots}
        self.ops: list[SimOp] = []
        self.cursor = dict.fromkeys(self.slots, 0)
        self.queues: dict[tuple, list] = defaultdict(list)  # channel -> [(mb, stage, arrival)]
        self.taken: dict[tuple, int] = defaultdict(int)

    def _heads(self, dst: Key, kind: str):
        for ch, q in self.queues.items():
            if ch[1] == dst and ch[2] == kind and self.taken[ch] < len(q):
                mb, stage, t = q[self.taken[ch]]
                yield mb, stage, t, ch

    def _ready(self, k: Key) -> list[tuple]:
        r, first = k[0], self.chunks[k][0]
        t0 = self.clock[k]
        room = self.holding[k] < self.limit.get(k, math.inf)
        ready = []
        if 0 in self.chunks[k] and room and self.entry_queue[(r, 0)]:
            ready.append((t0, "F", self.entry_queue[(r, 0)][0], 0, None))
        ready += [(max(t0, t), "F", mb, s, ch) for mb, s, t, ch in self._heads(k, "act") if room or s != first]
        if self.S - 1 in self.chunks[k]:
            tail = (r, self.S - 1)
            open_mbs = [m for m in self.fwd_end[tail] if m not in self.bwd_end[tail]]
            if open_mbs:
                m = min(open_mbs)
                ready.append((max(t0, self.fwd_end[tail][m]), "B", m, self.S - 1, None))
        ready += [(max(t0, t, self.fwd_end[(r, s)][mb]), "B", mb, s, ch) for mb, s, t, ch in self._heads(k, "grad")]
        if self.split and self.w_queue[k]:
            for s, m in (self.w_queue[k] if self.fixed is not None else self.w_queue[k][:1]):
                ready.append((max(t0, self.bwd_end[(r, s)][m]), "W", m, s, None))
        if self.fixed is not None:
            script = self.fixed[k]
            nxt = tuple(script[self.cursor[k]]) if self.cursor[k] < len(script) else None
            ready = [c for c in ready if (c[1], c[2], c[3]) == nxt]
        return ready

    def _emit(self, k: Key, choice: tuple) -> None:
        start, op, mb, s, ch = choice
        unit = (k[0], s)
        end = start + self.cost(unit, op, mb)
        self.busy[k] += end - start
        self.clock[k] = end
        self.order[k].append((op, mb, s) if self.interleaved else (op, mb))
        self.ops.append(SimOp(k, op, mb, start, end, s if self.interleaved else None))
        self.cursor[k] += 1
        if ch is not None:
            self.taken[ch] += 1
        first = self.chunks[k][0]
        if op == "W":
            self.w_queue[k].remove((s, mb))
            return
        if op == "F":
            if s == 0:
                self.entry_queue[unit].remove(mb)
            self.fwd_end[unit][mb] = end
            if s == first:
                self.holding[k] += 1
                self.peak[k] = max(self.peak[k], self.holding[k])
            nxt, kind = s + 1, "act"
        else:
            self.bwd_end[unit][mb] = end
            if s == first:
                self.holding[k] -= 1
            if self.split:
                self.w_queue[k].append((s, mb))
            nxt, kind = s - 1, "grad"
        if 0 <= nxt < self.S:
            peer = (self.plan.executor(nxt, mb), nxt)
            self.queues[(k, self.slot_of[peer], kind)].append((mb, nxt, end + self.comm(unit, peer, kind)))

    def run(self, sync_time, optimizer_time) -> SimResult:
        for _ in range(self.remaining):
            pick = None
            for k in self.slots:
                ready = self._ready(k)
                if not ready:
                    continue
                c = min(ready, key=lambda c: (c[0], _RANK[c[1]], c[2], c[3]))
                if pick is None or (c[0], _RANK[c[1]], k) < pick[0]:
                    pick = ((c[0], _RANK[c[1]], k), k, c)
            if pick is None:
                return SimResult(self.order, self.ops, math.inf, dict(self.clock), self.busy, self.peak, deadlock=True)
            self._emit(pick[1], pick[2])
        finish = {}
        for k in self.slots:
            tail = sum(sync_time((k[0], s)) for s in self.chunks[k]) if sync_time else 0.0
            finish[k] = self.clock[k] + tail
        fwd_done = {k: max((t for s in self.chunks[k] for t in self.fwd_end[(k[0], s)].values()), default=0.0)
                    for k in self.slots}
        return SimResult(self.order, self.ops, max(finish.values(), default=0.0) + optimizer_time, finish,
                         self.busy, self.peak, stage_forward_done=fwd_done)


def list_schedule(plan: HeteroParallelPlan, cost: CostFn, comm: CommFn, *, split_backward: bool = False,
                  inflight_limit: dict[Key, float] | None = None, sync_time: Callable[[Key], float] | None = None,
                  optimizer_time: float = 0.0, fixed: dict[Key, list[tuple]] | None = None) -> SimResult:
    """Greedy earliest-start schedule of F/B/(W) over the physical slots (module docstring).
    With ``fixed``, each slot follows its given ``(op, mb, stage)`` sequence and only the timing
    is computed."""
    return _Scheduler(plan, cost, comm, split_backward, inflight_limit, fixed).run(sync_time, optimizer_time)


def schedule_with_fallback(plan: HeteroParallelPlan, cost: CostFn, comm: CommFn, **kw) -> SimResult:
    """The in-flight-limited schedule -- for interleaved plans the faster of it and Megatron's
    static interleaved order -- or, if that deadlocks, the unlimited one (never deadlocks)."""
    no_limit = {plan.physical_key(g.replica, g.stage): math.inf for g in plan.stage_groups}
    unlimited = {**kw, "inflight_limit": no_limit}
    best = list_schedule(plan, cost, comm, **kw)
    static = megatron_interleaved_order(plan, kw.get("split_backward", False)) if plan.vpp > 1 else None
    if static is not None:
        alt = list_schedule(plan, cost, comm, fixed=static, **unlimited)
        if not alt.deadlock and (best.deadlock or alt.makespan < best.makespan):
            best = alt
    return best if not best.deadlock else list_schedule(plan, cost, comm, **unlimited)
