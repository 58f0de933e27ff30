"""Pipeline instruction IR run by the worker-side interpreter.

One instruction stream per physical (replica, stage) slot; every TP rank of a slot runs the
same stream.  Ops: ``F`` forward, ``B`` backward (input grad, or full backward), ``W`` weight
grad (zero-bubble split), ``SA``/``RA`` send/receive activation, ``SG``/``RG`` send/receive
gradient.  A communication instruction names its peer as a (replica, virtual stage) key; with
interleaving an instruction also carries its own virtual stage.

Safety conditions checked by ``validate`` (each direction of a rank pair is one FIFO channel,
sends never block): completeness (one F and one B per (stage, mb) on the executing slot, B
after F, W after B when split), per-channel receive order equal to send order, and deadlock
freedom by an earliest-start evaluation of the streams.

The JSON encoding of an instruction is ``[op, mb]``, ``[op, mb, r, s]`` or
``[op, mb, r|-1, s|-1, stage]`` -- the reference's format (``resihp/plan/ir.py:26-189``).
"""

from __future__ import annotations

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


@dataclass(frozen=True)
class Instr:
    op: Op
    mb: int
    peer: Key | None = None
    stage: int | None = None

    def stage_on(self, key: Key) -> int:
        """Virtual stage of this instruction inside the stream of slot ``key``."""
        return key[1] if self.stage is None else self.stage

    def to_json(self) -> list:
        head = [self.op.value, self.mb]
        if self.stage is None:
            return head + (list(self.peer) if self.peer is not None else [])
        return head + (list(self.peer) if self.peer is not None else [-1, -1]) + [self.stage]

    @staticmethod
    def from_json(d: list) -> "Instr":
        peer = (d[2], d[3]) if len(d) > 2 and d[2] >= 0 else None
        return Instr(Op(d[0]), d[1], peer, d[4] if len(d) > 4 else None)


Schedule = dict[Key, list[Instr]]


class ScheduleError(ValueError):
    pass


def compute_order_to_ir(plan: HeteroParallelPlan, order: dict[Key, list[tuple]]) -> Schedule:
    """Expand per-slot compute orders (``(op, mb)`` or ``(op, mb, stage)``) into streams with
    the receives before and the sends after each F / B."""
    last = plan.num_stages - 1
    out: Schedule = {}
    for key, entries in order.items():
        stream: list[Instr] = []
        for e in entries:
            op, mb = e[0], e[1]
            s = e[2] if len(e) > 2 else key[1]
            tag = s if plan.vpp > 1 else None
            if op == "F":
                if s > 0:
                    stream.append(Instr(Op.RECV_ACT, mb, (plan.executor(s - 1, mb), s - 1), tag))
                stream.append(Instr(Op.F, mb, None, tag))
                if s < last:
                    stream.append(Instr(Op.SEND_ACT, mb, (plan.executor(s + 1, mb), s + 1), tag))
            elif op == "B":
                if s < last:
                    stream.append(Instr(Op.RECV_GRAD, mb, (plan.executor(s + 1, mb), s + 1), tag))
                stream.append(Instr(Op.B, mb, None, tag))
                if s > 0:
                    stream.append(Instr(Op.SEND_GRAD, mb, (plan.executor(s - 1, mb), s - 1), tag))
            elif op == "W":
                stream.append(Instr(Op.W, mb, None, tag))
            else:
                raise ScheduleError(f"unknown compute op {op!r}")
        out[key] = stream
    return out


def schedule_to_json(schedule: Schedule) -> dict:
    return {f"{r},{s}": [i.to_json() for i in stream] for (r, s), stream in schedule.items()}


def schedule_from_json(d: dict) -> Schedule:
    out: Schedule = {}
    for k, stream in d.items():
        r, s = k.split(",")
        out[(int(r), int(s))] = [Instr.from_json(i) for i in stream]
    return out


def validate(plan: HeteroParallelPlan, schedule: Schedule, split_backward: bool = False) -> None:
    phys = lambda k: plan.physical_key(*k)  # noqa: E731
    for s in range(plan.num_stages):
        for m in range(plan.num_microbatches):
            key = phys((plan.executor(s, m), s))
            where: dict[Op, list[int]] = {op: [] for op in COMPUTE}
            for idx, ins in enumerate(schedule.get(key, [])):
                if ins.op in COMPUTE and ins.mb == m and ins.stage_on(key) == s:
                    where[ins.op].append(idx)
            if len(where[Op.F]) != 1 or len(where[Op.B]) != 1:
                raise ScheduleError(f"mb {m} stage {s}: expected exactly one F and one B on {key}")
            if where[Op.F][0] > where[Op.B][0]:
                raise ScheduleError(f"mb {m} stage {s}: B before F")
            if split_backward:
                if len(where[Op.W]) != 1 or where[Op.W][0] < where[Op.B][0]:
                    raise ScheduleError(f"mb {m} stage {s}: W missing or before B")
            elif where[Op.W]:
                raise ScheduleError(f"mb {m} stage {s}: unexpected W")
    for key, stream in schedule.items():
        for ins in stream:
            if ins.op in COMPUTE:
                s = ins.stage_on(key)
                if phys((plan.executor(s, ins.mb), s)) != key:
                    raise ScheduleError(f"{key} runs mb {ins.mb} of stage {s}, assigned to replica "
                                        f"{plan.executor(s, ins.mb)}")
    sent: dict[tuple, list[tuple[int, int]]] = {}
    got: dict[tuple, list[tuple[int, int]]] = {}
    for key, stream in schedule.items():
        for ins in stream:
            if ins.op in SENDS:
                sent.setdefault((key, phys(ins.peer), SENDS[ins.op]), []).append((ins.mb, ins.peer[1]))
            elif ins.op in RECVS:
                got.setdefault((phys(ins.peer), key, RECVS[ins.op]), []).append((ins.mb, ins.stage_on(key)))
    for ch in sent.keys() | got.keys():
        if sent.get(ch, []) != got.get(ch, []):
            raise ScheduleError(f"channel {ch}: send order {sent.get(ch)} != receive order {got.get(ch)}")
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
    """Earliest-start evaluation of fixed streams (DAG longest path): sends never block, a
    receive starts once its matching send finished plus the transfer time."""
    ptr = {k: 0 for k in schedule}
    clock = {k: 0.0 for k in schedule}
    arrivals: dict[tuple, float] = {}
    moved = True
    while moved:
        moved = False
        for key, stream in schedule.items():
            while ptr[key] < len(stream):
                ins = stream[ptr[key]]
                t0 = clock[key]
                if ins.op in RECVS:
                    tag = (phys(ins.peer), key, RECVS[ins.op], ins.mb, ins.stage_on(key))
                    if tag not in arrivals:
                        break
                    t0 = max(t0, arrivals[tag])
                t1 = t0 + duration(key, ins)
                if ins.op in SENDS:
                    arrivals[(key, phys(ins.peer), SENDS[ins.op], ins.mb, ins.peer[1])] = t1 + transfer(key, ins.peer,
                                                                                                       ins)
                clock[key] = t1
                ptr[key] += 1
                moved = True
    done = all(ptr[k] == len(s) for k, s in schedule.items())
    return StreamSimResult(done, dict(clock), max(clock.values(), default=0.0))
