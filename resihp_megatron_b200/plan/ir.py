"""Pipeline instruction IR, executed by the worker-side interpreter.

Each physical (replica, stage) slot runs one instruction stream; all TP ranks of the slot run
the same stream.  Ops: ``F`` forward, ``B`` backward (input gradient only when the backward is
split, else the full backward), ``W`` weight gradient (zero-bubble split), and the four
transfers ``SA``/``RA`` (send / receive activation) and ``SG``/``RG`` (send / receive gradient).
A transfer names its peer as a (replica, virtual stage) key; with interleaving every
instruction also carries its own virtual stage.

``validate`` proves a schedule safe under the runtime's channel model -- each direction between
two slots is one FIFO channel and sends never block:

* coverage: exactly one F and one B of every (stage, micro-batch) on the slot the plan assigns
  it to, B after F, and one W after B exactly when the backward is split;
* placement: no slot computes a (stage, micro-batch) assigned elsewhere;
* FIFO: on every channel the receive order equals the send order;
* progress: an earliest-start evaluation of all streams runs every instruction (no deadlock).

The JSON encoding of an instruction, ``[op, mb]``, ``[op, mb, r, s]`` or
``[op, mb, r|-1, s|-1, stage]``, is the reference's wire format (``resihp/plan/ir.py:26-189``).
"""

from __future__ import annotations

from collections import defaultdict, deque
from dataclasses import dataclass
from enum import Enum
from typing import Callable

from .hetero_plan import HeteroParallelPlan

Key = tuple[int, int]


class Op(str, Enum):
    F = "F"
    B = "B"
    W = "W"
    SEND_ACT = "SA"
    RECV_ACT = "RA"
    SEND_GRAD = "SG"
    RECV_GRAD = "RG"


COMPUTE = frozenset({Op.F, Op.B, Op.W})
SENDS = {Op.SEND_ACT: "act", Op.SEND_GRAD: "grad"}
RECVS = {Op.RECV_ACT: "act", Op.RECV_GRAD: "grad"}

# compute op -> (receive before it, offset of its source stage, send after it, offset of its target)
_WIRING = {"F": (Op.RECV_ACT, -1, Op.SEND_ACT, +1), "B": (Op.RECV_GRAD, +1, Op.SEND_GRAD, -1)}


@dataclass(frozen=True)
class Instr:
    op: Op
    mb: int
    peer: Key | None = None
    stage: int | None = None

    def stage_on(self, key: Key) -> int:
        """The virtual stage this instruction belongs to inside the stream of slot ``key``."""
        return self.stage if self.stage is not None else key[1]

    def to_json(self) -> list:
        enc = [self.op.value, self.mb]
        if self.peer is not None:
            enc.extend(self.peer)
        elif self.stage is not None:
            enc.extend((-1, -1))
        if self.stage is not None:
            enc.append(self.stage)
        return enc

    @classmethod
    def from_json(cls, d: list) -> "Instr":
        has_peer = len(d) >= 4 and d[2] >= 0
        return cls(Op(d[0]), d[1], (d[2], d[3]) if has_peer else None, d[4] if len(d) >= 5 else None)


Schedule = dict[Key, list[Instr]]


class ScheduleError(ValueError):
    pass


def compute_order_to_ir(plan: HeteroParallelPlan, order: dict[Key, list[tuple]]) -> Schedule:
    """Expand per-slot compute orders -- entries ``(op, mb)`` or ``(op, mb, stage)`` -- into
    instruction streams: a receive before and a send after every F and B that has a neighbour."""
    first, last = 0, plan.num_stages - 1
    streams: Schedule = {}
    for key, entries in order.items():
        out = streams.setdefault(key, [])
        for entry in entries:
            op, mb = entry[0], entry[1]
            s = entry[2] if len(entry) > 2 else key[1]
            tag = s if plan.vpp > 1 else None
            if op == "W":
                out.append(Instr(Op.W, mb, None, tag))
                continue
            if op not in _WIRING:
                raise ScheduleError(f"unknown compute op {op!r}")
            recv, src, send, dst = _WIRING[op]
            if first <= s + src <= last:
                out.append(Instr(recv, mb, (plan.executor(s + src, mb), s + src), tag))
            out.append(Instr(Op(op), mb, None, tag))
            if first <= s + dst <= last:
                out.append(Instr(send, mb, (plan.executor(s + dst, mb), s + dst), tag))
    return streams


def schedule_to_json(schedule: Schedule) -> dict:
    return {"%d,%d" % key: [i.to_json() for i in stream] for key, stream in schedule.items()}


def schedule_from_json(d: dict) -> Schedule:
    def key(text: str) -> Key:
        r, s = map(int, text.split(","))
        return r, s

    return {key(k): list(map(Instr.from_json, stream)) for k, stream in d.items()}


def _check_coverage(plan: HeteroParallelPlan, schedule: Schedule, split: bool, phys) -> None:
    positions: dict[tuple, dict[Op, list[int]]] = defaultdict(lambda: defaultdict(list))
    for key, stream in schedule.items():
        for idx, ins in enumerate(stream):
            if ins.op in COMPUTE:
                positions[(key, ins.stage_on(key), ins.mb)][ins.op].append(idx)
    for s in range(plan.num_stages):
        for m in range(plan.num_microbatches):
            key = phys((plan.executor(s, m), s))
            at = positions.get((key, s, m), {})
            f, b, w = at.get(Op.F, []), at.get(Op.B, []), at.get(Op.W, [])
            if len(f) != 1 or len(b) != 1:
                raise ScheduleError(f"mb {m} stage {s}: expected exactly one F and one B on {key}")
            if b[0] < f[0]:
                raise ScheduleError(f"mb {m} stage {s}: B before F")
            if split and (len(w) != 1 or w[0] < b[0]):
                raise ScheduleError(f"mb {m} stage {s}: W missing or before B")
            if not split and w:
                raise ScheduleError(f"mb {m} stage {s}: unexpected W")


def _check_placement(plan: HeteroParallelPlan, schedule: Schedule, phys) -> None:
    for key, stream in schedule.items():
        for ins in filter(lambda i: i.op in COMPUTE, stream):
            s = ins.stage_on(key)
            owner = plan.executor(s, ins.mb)
            if phys((owner, s)) != key:
                raise ScheduleError(f"{key} runs mb {ins.mb} of stage {s}, assigned to replica {owner}")


def _check_fifo(schedule: Schedule, phys) -> None:
    posted, taken = defaultdict(list), defaultdict(list)
    for key, stream in schedule.items():
        for ins in stream:
            if ins.op in SENDS:
                posted[(key, phys(ins.peer), SENDS[ins.op])].append((ins.mb, ins.peer[1]))
            elif ins.op in RECVS:
                taken[(phys(ins.peer), key, RECVS[ins.op])].append((ins.mb, ins.stage_on(key)))
    for channel in set(posted) | set(taken):
        if posted.get(channel, []) != taken.get(channel, []):
            raise ScheduleError(f"channel {channel}: send order {posted.get(channel)} != receive order "
                                f"{taken.get(channel)}")


def validate(plan: HeteroParallelPlan, schedule: Schedule, split_backward: bool = False) -> None:
    """Raise ``ScheduleError`` unless ``schedule`` is complete, FIFO-consistent and deadlock free."""

    def phys(k: Key) -> Key:
        return plan.physical_key(*k)

    _check_coverage(plan, schedule, split_backward, phys)
    _check_placement(plan, schedule, phys)
    _check_fifo(schedule, phys)
    if not stream_simulation(schedule, phys=phys).complete:
        raise ScheduleError("schedule deadlocks")


@dataclass
class StreamSimResult:
    complete: bool
    finish: dict[Key, float]
    makespan: float


def _unit(key, ins) -> float:
    return 1.0 if ins.op in COMPUTE else 0.0


def stream_simulation(schedule: Schedule, duration: Callable = _unit, transfer: Callable = lambda s, d, i: 0.0,
                      phys: Callable = lambda k: k) -> StreamSimResult:
    """Earliest-start evaluation of fixed streams (the longest path of their DAG).  A stream
    advances until it reaches a receive whose message was not sent yet; a send wakes the
    receiving stream.  Sends never block; a receive starts at the later of its stream's clock
    and its message's arrival (send end + ``transfer``)."""
    pc = dict.fromkeys(schedule, 0)
    now = dict.fromkeys(schedule, 0.0)
    arrived: dict[tuple, float] = {}
    waiting: dict[tuple, Key] = {}
    ready = deque(schedule)
    while ready:
        key = ready.popleft()
        stream = schedule[key]
        while pc[key] < len(stream):
            ins = stream[pc[key]]
            start = now[key]
            if ins.op in RECVS:
                msg = (phys(ins.peer), key, RECVS[ins.op], ins.mb, ins.stage_on(key))
                if msg not in arrived:
                    waiting[msg] = key
                    break
                start = max(start, arrived[msg])
            end = start + duration(key, ins)
            if ins.op in SENDS:
                dst = phys(ins.peer)
                msg = (key, dst, SENDS[ins.op], ins.mb, ins.peer[1])
                arrived[msg] = end + transfer(key, ins.peer, ins)
                if waiting.get(msg) is not None:
                    ready.append(waiting.pop(msg))
            now[key] = end
            pc[key] += 1
    complete = all(pc[k] == len(s) for k, s in schedule.items())
    return StreamSimResult(complete, dict(now), max(now.values(), default=0.0))
