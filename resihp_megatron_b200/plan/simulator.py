"""List-scheduling pipeline simulator, shared by the planner and the fail-slow detector.

Given a plan and a cost model it builds a concrete compute order per physical slot
(1F1B-like with an in-flight limit, optional zero-bubble W filling), the op timings, each
slot's peak number of in-flight micro-batches, and the makespan.  Message channels are
physical (src slot, dst slot, kind) FIFOs consumed strictly in send order -- the NCCL-safety
discipline -- so every order it produces converts to a valid IR (``ir.compute_order_to_ir``).

Scheduling rule: repeatedly pick, over all slots, the candidate op with the earliest start
time (ties: backward before forward before weight-grad, then lower micro-batch, then lower
stage, then slot key).  Candidates of a slot: the next entry forward (if under the in-flight
limit), the heads of the slot's incoming activation channels, the oldest pending last-stage
backward, the heads of incoming gradient channels, and queued W ops.
Semantics follow ``resihp/plan/simulator.py:45-251`` of the reference.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable

from .hetero_plan import HeteroParallelPlan

Key = tuple[int, int]
CostFn = Callable[[Key, str, int], float]
CommFn = Callable[[Key, Key, str], float]

_PRIORITY = {"B": 0, "F": 1, "W": 2}


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
    """Micro-batches a physical slot may hold between its first forward and last backward.

    Plain 1F1B: warm-up depth ``P - p``, scaled up by the slot's share of its stage's
    micro-batches (a slot that absorbs migrated micro-batches needs proportionally more
    warm-up).  Interleaved: only the pipeline entry is limited, to the interleaved warm-up
    depth, which bounds every slot (a per-slot limit could block a chunk-0 message at a
    channel head in front of a chunk-1 message)."""
    P, v = plan.num_physical_stages, plan.vpp
    lim: dict[Key, float] = {}
    for g in plan.stage_groups:
        r, p = plan.physical_key(g.replica, g.stage)
        if v == 1:
            share = len(plan.microbatches_of(r, p)) * plan.num_replicas / plan.num_microbatches
            lim[(r, p)] = max(1, math.ceil((P - p) * max(1.0, share)))
        else:
            lim[(r, p)] = (math.ceil(((P - 1) * 2 + (v - 1) * P) / v) + 1) if p == 0 else math.inf
    return lim


def megatron_interleaved_order(plan: HeteroParallelPlan, split_backward: bool = False):
    """The static interleaved 1F1B order per physical slot: forwards in groups of ``P``
    micro-batches chunk by chunk, backwards with chunks reversed, warm-up
    ``(P - p - 1) * 2 + (v - 1) * P``; with a split backward each W follows its B.  ``None``
    when the chunks of a slot run different micro-batch sets."""
    P, v = plan.num_physical_stages, plan.vpp
    out: dict[Key, list[tuple]] = {}
    for g in plan.stage_groups:
        r, p = plan.physical_key(g.replica, g.stage)
        if (r, p) in out:
            continue
        mbs = plan.microbatches_of(r, p)
        for c in range(v):
            if plan.group(r, p + c * P) is None or plan.microbatches_of(r, p + c * P) != mbs:
                return None
        n = len(mbs)

        def nth(k: int, backward: bool) -> tuple[int, int]:
            base = (k // (P * v)) * P
            width = min(P, n - base)
            c, i = divmod(k - base * v, width)
            chunk = (v - 1 - c) if backward else c
            return mbs[base + i], chunk * P + p

        total = n * v
        warm = min(total, (P - p - 1) * 2 + (v - 1) * P)
        seq: list[tuple] = [("F",) + nth(k, False) for k in range(warm)]

        def push_back(i: int) -> None:
            mb, s = nth(i, True)
            seq.append(("B", mb, s))
            if split_backward:
                seq.append(("W", mb, s))

        for i in range(total - warm):
            seq.append(("F",) + nth(warm + i, False))
            push_back(i)
        for i in range(total - warm, total):
            push_back(i)
        out[(r, p)] = seq
    return out


class _Channels:
    """FIFO message channels keyed by (src slot, dst slot, kind)."""

    def __init__(self):
        self.msgs: dict[tuple, list[tuple[int, int, float]]] = {}
        self.head: dict[tuple, int] = {}

    def push(self, ch: tuple, mb: int, stage: int, t: float) -> None:
        self.msgs.setdefault(ch, []).append((mb, stage, t))
        self.head.setdefault(ch, 0)

    def heads_into(self, dst: Key, kind: str):
        for ch, q in self.msgs.items():
            h = self.head[ch]
            if ch[1] == dst and ch[2] == kind and h < len(q):
                yield q[h] + (ch,)

    def pop(self, ch: tuple) -> None:
        self.head[ch] += 1


def list_schedule(plan: HeteroParallelPlan, cost: CostFn, comm: CommFn, *, split_backward: bool = False,
                  inflight_limit: dict[Key, float] | None = None, sync_time: Callable[[Key], float] | None = None,
                  optimizer_time: float = 0.0, fixed: dict[Key, list[tuple]] | None = None) -> SimResult:
    """Greedy earliest-start scheduling of F/B/(W) over physical slots (see module docstring).
    With ``fixed`` each slot follows the given ``(op, mb, stage)`` sequence and only timing is
    computed."""
    S, M = plan.num_stages, plan.num_microbatches
    interleaved = plan.vpp > 1
    units = [(g.replica, g.stage) for g in plan.stage_groups]
    slot_of = {u: plan.physical_key(*u) for u in units}
    slots = sorted(set(slot_of.values()))
    chunks = {k: sorted(u[1] for u in units if slot_of[u] == k) for k in slots}
    limit = inflight_limit if inflight_limit is not None else default_inflight_limit(plan)
    todo_f0 = {u: [m for m in range(M) if plan.executor(u[1], m) == u[0]] for u in units}
    n_ops = sum(len(v) for v in todo_f0.values()) * (3 if split_backward else 2)
    f_end: dict[Key, dict[int, float]] = {u: {} for u in units}
    b_end: dict[Key, dict[int, float]] = {u: {} for u in units}
    w_queue: dict[Key, list[tuple[int, int]]] = {k: [] for k in slots}
    free = {k: 0.0 for k in slots}
    busy = {k: 0.0 for k in slots}
    inflight = {k: 0 for k in slots}
    peak = {k: 0 for k in slots}
    order: dict[Key, list[tuple]] = {k: [] for k in slots}
    ops: list[SimOp] = []
    chans = _Channels()
    cursor = {k: 0 for k in slots} if fixed is not None else None

    def candidates(k: Key) -> list[tuple]:
        r, first = k[0], chunks[k][0]
        under = inflight[k] < limit.get(k, math.inf)
        out = []
        if 0 in chunks[k] and todo_f0[(r, 0)] and under:
            out.append((free[k], "F", todo_f0[(r, 0)][0], 0, None))
        for mb, s, t, ch in chans.heads_into(k, "act"):
            if s != first or under:
                out.append((max(free[k], t), "F", mb, s, ch))
        if S - 1 in chunks[k]:
            u = (r, S - 1)
            pending = sorted(m for m in f_end[u] if m not in b_end[u])
            if pending:
                out.append((max(free[k], f_end[u][pending[0]]), "B", pending[0], S - 1, None))
        for mb, s, t, ch in chans.heads_into(k, "grad"):
            out.append((max(free[k], t, f_end[(r, s)][mb]), "B", mb, s, ch))
        if split_backward and w_queue[k]:
            queued = w_queue[k] if fixed is not None else w_queue[k][:1]
            for s, m in queued:
                out.append((max(free[k], b_end[(r, s)][m]), "W", m, s, None))
        if fixed is not None:
            seq = fixed[k]
            want = tuple(seq[cursor[k]]) if cursor[k] < len(seq) else None
            out = [c for c in out if want is not None and (c[1], c[2], c[3]) == want]
        return out

    for _ in range(n_ops):
        best = None
        for k in slots:
            cands = candidates(k)
            if not cands:
                continue
            c = min(cands, key=lambda c: (c[0], _PRIORITY[c[1]], c[2], c[3]))
            rank = (c[0], _PRIORITY[c[1]], k)
            if best is None or rank < best[0]:
                best = (rank, k, c)
        if best is None:
            return SimResult(order, ops, math.inf, dict(free), busy, peak, deadlock=True)
        _, k, (start, op, mb, s, ch) = best
        u = (k[0], s)
        end = start + cost(u, op, mb)
        busy[k] += end - start
        free[k] = end
        order[k].append((op, mb, s) if interleaved else (op, mb))
        ops.append(SimOp(k, op, mb, start, end, s if interleaved else None))
        if cursor is not None:
            cursor[k] += 1
        if ch is not None:
            chans.pop(ch)
        if op == "F":
            if s == 0:
                todo_f0[u].remove(mb)
            f_end[u][mb] = end
            if s == chunks[k][0]:
                inflight[k] += 1
                peak[k] = max(peak[k], inflight[k])
            if s < S - 1:
                dst = (plan.executor(s + 1, mb), s + 1)
                chans.push((k, slot_of[dst], "act"), mb, s + 1, end + comm(u, dst, "act"))
        elif op == "B":
            b_end[u][mb] = end
            if s == chunks[k][0]:
                inflight[k] -= 1
            if split_backward:
                w_queue[k].append((s, mb))
            if s > 0:
                dst = (plan.executor(s - 1, mb), s - 1)
                chans.push((k, slot_of[dst], "grad"), mb, s - 1, end + comm(u, dst, "grad"))
        else:
            w_queue[k].remove((s, mb))

    finish = {k: free[k] + (sum(sync_time((k[0], s)) for s in chunks[k]) if sync_time else 0.0) for k in slots}
    fwd_done = {k: max((t for s in chunks[k] for t in f_end[(k[0], s)].values()), default=0.0) for k in slots}
    return SimResult(order, ops, max(finish.values(), default=0.0) + optimizer_time, finish, busy, peak,
                     stage_forward_done=fwd_done)


def schedule_with_fallback(plan: HeteroParallelPlan, cost: CostFn, comm: CommFn, **kw) -> SimResult:
    """The in-flight-limited schedule (for interleaved plans also the static interleaved
    order, whichever the simulation finds faster); unlimited in-flight -- always deadlock
    free -- when the limited one deadlocks."""
    unlimited = {plan.physical_key(g.replica, g.stage): math.inf for g in plan.stage_groups}
    res = list_schedule(plan, cost, comm, **kw)
    if plan.vpp > 1:
        fixed = megatron_interleaved_order(plan, kw.get("split_backward", False))
        if fixed is not None:
            alt = list_schedule(plan, cost, comm, fixed=fixed, **{**kw, "inflight_limit": unlimited})
            if not alt.deadlock and (res.deadlock or alt.makespan < res.makespan):
                res = alt
    if not res.deadlock:
        return res
    return list_schedule(plan, cost, comm, **{**kw, "inflight_limit": unlimited})
