"""Worker-side interpreter of the pipeline IR (one stream per (replica, stage) slot).

Compute goes through a ``StageExecutor`` (the float64 reference model on CPU; the GPU model of
``models/`` through ``runtime/gpu_executor.py``); communication goes through ``P2PEngine`` with
heterogeneous-TP routing.  Sends are posted non-blocking and waited at the end of the iteration,
which is what the IR validator assumes.  Progress (op index, in-collective flag) is reported on
every instruction for hang detection, and fault-injection hooks fire at ``forward`` /
``backward``.  (Reference: ``resihp/runtime/interpreter.py:23-214``.)
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
    """``stage`` is the virtual stage (model chunk) the instruction belongs to."""

    def begin_iteration(self, iteration: int) -> None: ...
    def n_rows(self, mb: int) -> int: ...
    def forward(self, mb: int, inp: torch.Tensor | None, stage: int) -> torch.Tensor | None: ...
    def backward(self, mb: int, grad: torch.Tensor | None, stage: int) -> torch.Tensor | None: ...
    def weight_backward(self, mb: int, stage: int) -> None: ...


class RefStageExecutor:
    def __init__(self, cfg: RefModelConfig, sampler: IndexAddressableSampler, module, plan: HeteroParallelPlan,
                 replica: int, stage: int, rank: int, weight_grad_store=None, timer=None):
        self.cfg = cfg
        self.sampler = sampler
        self.module = module
        self.modules: dict[int, RefStage] = getattr(module, "chunks", None) or {stage: module}
        self.plan = plan
        self.group = plan.group(replica, stage)
        self.cp_index = self.group.slice_of(plan.world[rank])
        self.ranks = plan.slice_ranks(self.group, self.cp_index)
        self.rank = rank
        self.num_stages = plan.num_stages
        self.sp = plan.sequence_parallel and self.group.tp > 1
        self.iteration = -1
        self.saved: dict[tuple[int, int], tuple] = {}
        self.loss_sum = 0.0
        self._mbs: dict[int, MicroBatch] = {}
        self.wgs = weight_grad_store
        self.timer = timer
        self.fwd_docs: dict[int, list[int]] = {}

    def begin_iteration(self, iteration: int) -> None:
        self.iteration = iteration
        self.saved.clear()
        self._mbs.clear()
        self.loss_sum = 0.0
        self.fwd_docs = {}

    def timing_samples(self) -> list[tuple[float, float, float]]:
        """(tokens, sum of squared doc lengths, forward seconds over local chunks) per micro-batch."""
        if self.timer is None:
            return []
        secs: dict[int, float] = {}
        for rec in self.timer.collect():
            if rec.op == "F" and rec.iteration == self.iteration and rec.mb in self.fwd_docs:
                secs[rec.mb] = secs.get(rec.mb, 0.0) + rec.seconds
        return [(float(sum(self.fwd_docs[mb])), float(sum(d * d for d in self.fwd_docs[mb])), s)
                for mb, s in secs.items()]

    def _timed(self, op: str, mb: int):
        return self.timer.time(self.iteration, op, mb) if self.timer is not None else nullcontext()

    def _mb(self, mb: int) -> MicroBatch:
        m = self._mbs.get(mb)
        if m is None:
            m = microbatch(self.cfg, self.sampler, self.iteration, mb)
            if self.cfg.device != "cpu":
                dev = self.cfg.device
                m = MicroBatch(m.x.to(dev), m.y.to(dev), m.mask.to(dev), m.doc_lengths)
            self._mbs[mb] = m
        return m

    def _chunk(self, mb: int) -> tuple[int, int]:
        """Token rows of this rank's context-parallel chunk of the micro-batch."""
        return even_split(self._mb(mb).x.shape[0], self.group.cp)[self.cp_index]

    def n_rows(self, mb: int) -> int:
        a, b = self._chunk(mb)
        return b - a

    def _rows(self, mb: int) -> tuple[int, int]:
        a, b = self._chunk(mb)
        if not self.sp:
            return a, b
        s, e = local_rows(b - a, self.ranks, self.rank)
        return a + s, a + e

    def forward(self, mb: int, inp: torch.Tensor | None, stage: int) -> torch.Tensor | None:
        first, last = stage == 0, stage == self.num_stages - 1
        s, e = self._rows(mb)
        x = self._mb(mb).x[s:e].clone() if first else inp.detach().requires_grad_(True)
        with self._timed("F", mb):
            out = self.modules[stage](x)
            if last:
                m = self._mb(mb)
                loss = token_loss(out, m.y[s:e], m.mask[s:e])
        self.fwd_docs[mb] = self._mb(mb).doc_lengths
        if last:
            self.loss_sum += loss.item()
            self.saved[(stage, mb)] = (x, loss)
            return None
        self.saved[(stage, mb)] = (x, out)
        return out.detach()

    def backward(self, mb: int, grad: torch.Tensor | None, stage: int) -> torch.Tensor | None:
        first, last = stage == 0, stage == self.num_stages - 1
        x, out = self.saved.pop((stage, mb))
        if self.wgs is not None and hasattr(self.wgs, "backward_input"):
            with self._timed("B", mb):
                return self.wgs.backward_input((stage, mb), out, None if last else grad, None if first else x)
        ctx = self.wgs.deferring((stage, mb)) if self.wgs is not None else nullcontext()
        with ctx, self._timed("B", mb):
            if last:
                out.backward()
            else:
                torch.autograd.backward(out, grad)
        return None if first else x.grad

    def weight_backward(self, mb: int, stage: int) -> None:
        if self.wgs is not None:
            self.wgs.compute((stage, mb))


def message_tag(mb: int, kind: str, dst_stage: int) -> int:
    return (mb * 2 + (0 if kind == "act" else 1)) * 256 + dst_stage


class Interpreter:
    def __init__(self, plan: HeteroParallelPlan, stream: list[Instr], executor: StageExecutor, p2p: P2PEngine,
                 replica: int, stage: int, row_shape: tuple[int, ...], dtype: torch.dtype, tp_group=None,
                 progress=None, hook=None):
        self.plan = plan
        self.stream = stream
        self.executor = executor
        self.p2p = p2p
        self.key = (replica, stage)
        self.group = plan.group(replica, stage)
        # activations stay inside a context-parallel chunk: slice i only talks to slice i
        self.cp_index = self.group.slice_of(plan.world[p2p.rank])
        self.ranks = plan.slice_ranks(self.group, self.cp_index)
        self.row_shape = row_shape
        self.dtype = dtype
        self.tp_group = tp_group
        self.sp = plan.sequence_parallel
        self.progress = progress or (lambda **kw: None)
        self.hook = hook or (lambda it, phase: None)

    def peer_ranks(self, peer: tuple[int, int]) -> tuple[int, ...]:
        return self.plan.slice_ranks(self.plan.group(*peer), self.cp_index)

    def _recv(self, mb: int, kind: str, stage: int, peer) -> torch.Tensor:
        ex = self.executor
        return self.p2p.recv(ex.n_rows(mb), self.row_shape, self.dtype, self.peer_ranks(peer), self.ranks, self.sp,
                             message_tag(mb, kind, stage), self.tp_group)

    def _send(self, t: torch.Tensor, mb: int, kind: str, peer) -> list:
        return self.p2p.send(t, self.ranks, self.peer_ranks(peer), self.executor.n_rows(mb), self.sp,
                             message_tag(mb, kind, peer[1]))

    def run(self, iteration: int) -> None:
        ex = self.executor
        ex.begin_iteration(iteration)
        acts: dict = {}
        grads: dict = {}
        outs: dict = {}
        igrads: dict = {}
        sends: list = []
        for i, ins in enumerate(self.stream):
            self.progress(iteration=iteration, phase=f"{ins.op.value}{ins.mb}", op_seq=i,
                          in_collective=ins.op in (Op.RECV_ACT, Op.RECV_GRAD))
            mb, s = ins.mb, ins.stage_on(self.key)
            k = (s, mb)
            if ins.op == Op.RECV_ACT:
                acts[k] = self._recv(mb, "act", s, ins.peer)
            elif ins.op == Op.F:
                self.hook(iteration, "forward")
                out = ex.forward(mb, acts.pop(k, None), s)
                if out is not None:
                    outs[k] = out
            elif ins.op == Op.SEND_ACT:
                sends += self._send(outs.pop(k), mb, "act", ins.peer)
            elif ins.op == Op.RECV_GRAD:
                grads[k] = self._recv(mb, "grad", s, ins.peer)
            elif ins.op == Op.B:
                self.hook(iteration, "backward")
                g = ex.backward(mb, grads.pop(k, None), s)
                if g is not None:
                    igrads[k] = g
            elif ins.op == Op.SEND_GRAD:
                sends += self._send(igrads.pop(k), mb, "grad", ins.peer)
            elif ins.op == Op.W:
                ex.weight_backward(mb, s)
        self.p2p.wait_sends(sends)
