"""Worker-side interpreter of the pipeline IR (one instruction stream per (replica, stage) slot).

Compute is delegated to a ``StageExecutor`` -- the float64 reference model on the CPU, the GPU
decoder through ``runtime/gpu_executor.py`` -- and transfers to the ``P2PEngine`` with
heterogeneous-TP routing.  Sends are posted non-blocking and waited for at the end of the
iteration, the channel model the IR validator proves safe.  Every instruction reports progress
(op index, whether it waits on a peer) for hang detection, and fault-injection hooks fire at
``forward`` and ``backward``.
Parity: ``resihp/runtime/interpreter.py:23-214`` (same ops, tags and progress reports).
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Protocol

import torch

from ..comm.p2p import P2PEngine, local_rows
from ..plan.hetero_plan import HeteroParallelPlan
from ..plan.ir import Instr, Op
from ..state.rng_data import IndexAddressableSampler
from ..utils.intervals import even_split
from .reference_model import MicroBatch, RefModelConfig, RefStage, microbatch, token_loss


class StageExecutor(Protocol):
    """``stage`` is the virtual stage (model chunk) an instruction belongs to."""

    def begin_iteration(self, iteration: int) -> None: ...
    def n_rows(self, mb: int) -> int: ...
    def forward(self, mb: int, inp: torch.Tensor | None, stage: int) -> torch.Tensor | None: ...
    def backward(self, mb: int, grad: torch.Tensor | None, stage: int) -> torch.Tensor | None: ...
    def weight_backward(self, mb: int, stage: int) -> None: ...


class RefStageExecutor:
    """Runs the reference model's chunks of one slot on its rank's rows of each micro-batch."""

    def __init__(self, cfg: RefModelConfig, sampler: IndexAddressableSampler, module, plan: HeteroParallelPlan,
                 replica: int, stage: int, rank: int, weight_grad_store=None, timer=None):
        self.cfg, self.sampler, self.module, self.plan, self.rank = cfg, sampler, module, plan, rank
        self.modules: dict[int, RefStage] = getattr(module, "chunks", None) or {stage: module}
        self.group = plan.group(replica, stage)
        self.cp_index = self.group.slice_of(plan.world[rank])
        self.ranks = plan.slice_ranks(self.group, self.cp_index)
        self.num_stages = plan.num_stages
        self.sp = plan.sequence_parallel and self.group.tp > 1
        self.wgs, self.timer = weight_grad_store, timer
        self.iteration = -1
        self.loss_sum = 0.0
        self.saved: dict[tuple[int, int], tuple] = {}
        self.fwd_docs: dict[int, list[int]] = {}
        self._batches: dict[int, MicroBatch] = {}

    def begin_iteration(self, iteration: int) -> None:
        self.iteration, self.loss_sum = iteration, 0.0
        self.saved.clear()
        self._batches.clear()
        self.fwd_docs = {}

    def timing_samples(self) -> list[tuple[float, float, float]]:
        """Per micro-batch: (tokens, sum of squared document lengths, forward seconds over this
        slot's chunks)."""
        if self.timer is None:
            return []
        seconds: dict[int, float] = {}
        for rec in self.timer.collect():
            if rec.op == "F" and rec.iteration == self.iteration and rec.mb in self.fwd_docs:
                seconds[rec.mb] = seconds.get(rec.mb, 0.0) + rec.seconds
        out = []
        for mb, secs in seconds.items():
            docs = self.fwd_docs[mb]
            out.append((float(sum(docs)), float(sum(d * d for d in docs)), secs))
        return out

    def _timed(self, op: str, mb: int):
        return nullcontext() if self.timer is None else self.timer.time(self.iteration, op, mb)

    def _batch(self, mb: int) -> MicroBatch:
        if mb not in self._batches:
            b = microbatch(self.cfg, self.sampler, self.iteration, mb)
            if self.cfg.device != "cpu":
                d = self.cfg.device
                b = MicroBatch(b.x.to(d), b.y.to(d), b.mask.to(d), b.doc_lengths)
            self._batches[mb] = b
        return self._batches[mb]

    def _cp_rows(self, mb: int) -> tuple[int, int]:
        """Token rows of this rank's context-parallel chunk."""
        return even_split(self._batch(mb).x.shape[0], self.group.cp)[self.cp_index]

    def n_rows(self, mb: int) -> int:
        lo, hi = self._cp_rows(mb)
        return hi - lo

    def _rows(self, mb: int) -> tuple[int, int]:
        lo, hi = self._cp_rows(mb)
        if not self.sp:
            return lo, hi
        a, b = local_rows(hi - lo, self.ranks, self.rank)
        return lo + a, lo + b

    def forward(self, mb: int, inp: torch.Tensor | None, stage: int) -> torch.Tensor | None:
        lo, hi = self._rows(mb)
        batch = self._batch(mb)
        x = batch.x[lo:hi].clone() if stage == 0 else inp.detach().requires_grad_(True)
        last = stage == self.num_stages - 1
        with self._timed("F", mb):
            y = self.modules[stage](x)
            if last:
                y = token_loss(y, batch.y[lo:hi], batch.mask[lo:hi])
        self.fwd_docs[mb] = batch.doc_lengths
        self.saved[(stage, mb)] = (x, y)
        if last:
            self.loss_sum += y.item()
            return None
        return y.detach()

    def backward(self, mb: int, grad: torch.Tensor | None, stage: int) -> torch.Tensor | None:
        x, y = self.saved.pop((stage, mb))
        first, last = stage == 0, stage == self.num_stages - 1
        upstream = None if last else grad
        if self.wgs is not None and hasattr(self.wgs, "backward_input"):
            with self._timed("B", mb):
                return self.wgs.backward_input((stage, mb), y, upstream, None if first else x)
        defer = self.wgs.deferring((stage, mb)) if self.wgs is not None else nullcontext()
        with defer, self._timed("B", mb):
            torch.autograd.backward(y, upstream)
        return None if first else x.grad

    def weight_backward(self, mb: int, stage: int) -> None:
        if self.wgs is not None:
            self.wgs.compute((stage, mb))


def message_tag(mb: int, kind: str, dst_stage: int) -> int:
    """Tag of an activation / gradient message: micro-batch, kind and destination stage."""
    return ((2 * mb + (kind != "act")) << 8) + dst_stage


class Interpreter:
    def __init__(self, plan: HeteroParallelPlan, stream: list[Instr], executor: StageExecutor, p2p: P2PEngine,
                 replica: int, stage: int, row_shape: tuple[int, ...], dtype: torch.dtype, tp_group=None,
                 progress=None, hook=None):
        self.plan, self.stream, self.executor, self.p2p = plan, stream, executor, p2p
        self.key = (replica, stage)
        self.group = plan.group(replica, stage)
        # activations never leave a context-parallel chunk: slice i only talks to slice i
        self.cp_index = self.group.slice_of(plan.world[p2p.rank])
        self.ranks = plan.slice_ranks(self.group, self.cp_index)
        self.row_shape, self.dtype, self.tp_group = row_shape, dtype, tp_group
        self.sp = plan.sequence_parallel
        self.progress = progress if progress is not None else (lambda **kw: None)
        self.hook = hook if hook is not None else (lambda it, phase: None)
        self._ops = {Op.RECV_ACT: self._recv_act, Op.F: self._forward, Op.SEND_ACT: self._send_act,
                     Op.RECV_GRAD: self._recv_grad, Op.B: self._backward, Op.SEND_GRAD: self._send_grad,
                     Op.W: self._weight}

    def peer_ranks(self, peer: tuple[int, int]) -> tuple[int, ...]:
        return self.plan.slice_ranks(self.plan.group(*peer), self.cp_index)

    def _receive(self, mb: int, kind: str, stage: int, peer) -> torch.Tensor:
        return self.p2p.recv(self.executor.n_rows(mb), self.row_shape, self.dtype, self.peer_ranks(peer), self.ranks,
                             self.sp, message_tag(mb, kind, stage), self.tp_group)

    def _post(self, t: torch.Tensor, mb: int, kind: str, peer) -> None:
        self._sends += self.p2p.send(t, self.ranks, self.peer_ranks(peer), self.executor.n_rows(mb), self.sp,
                                     message_tag(mb, kind, peer[1]))

    # one handler per op; ``slot`` is (virtual stage, micro-batch)
    def _recv_act(self, ins: Instr, slot, it: int) -> None:
        self._box["act"][slot] = self._receive(ins.mb, "act", slot[0], ins.peer)

    def _forward(self, ins: Instr, slot, it: int) -> None:
        self.hook(it, "forward")
        out = self.executor.forward(ins.mb, self._box["act"].pop(slot, None), slot[0])
        if out is not None:
            self._box["out"][slot] = out

    def _send_act(self, ins: Instr, slot, it: int) -> None:
        self._post(self._box["out"].pop(slot), ins.mb, "act", ins.peer)

    def _recv_grad(self, ins: Instr, slot, it: int) -> None:
        self._box["grad"][slot] = self._receive(ins.mb, "grad", slot[0], ins.peer)

    def _backward(self, ins: Instr, slot, it: int) -> None:
        self.hook(it, "backward")
        g = self.executor.backward(ins.mb, self._box["grad"].pop(slot, None), slot[0])
        if g is not None:
            self._box["igrad"][slot] = g

    def _send_grad(self, ins: Instr, slot, it: int) -> None:
        self._post(self._box["igrad"].pop(slot), ins.mb, "grad", ins.peer)

    def _weight(self, ins: Instr, slot, it: int) -> None:
        self.executor.weight_backward(ins.mb, slot[0])

    def run(self, iteration: int) -> None:
        self.executor.begin_iteration(iteration)
        self._box = {"act": {}, "out": {}, "grad": {}, "igrad": {}}
        self._sends: list = []
        for index, ins in enumerate(self.stream):
            waiting = ins.op in (Op.RECV_ACT, Op.RECV_GRAD)
            self.progress(iteration=iteration, phase=f"{ins.op.value}{ins.mb}", op_seq=index, in_collective=waiting)
            self._ops[ins.op](ins, (ins.stage_on(self.key), ins.mb), iteration)
        self.p2p.wait_sends(self._sends)
