"""One generation's dynamic hybrid-parallel data plane on the reference model: heterogeneous
TP, uneven PP, stage-level micro-batch migration, CP chunking, zero-bubble W and interleaved
chunks.

``run_iteration`` interprets this slot's IR stream, runs the shard-aligned gradient sync of
every local chunk, reduces the fp8 amax of every layer (MAX over all ranks) and updates its
history, divides gradients by the global token count, all-reduces the loss, and (first rank of
the group only) reports per-micro-batch forward timings for fail-slow detection.
``channel_specs`` derives one 2-rank group per direction of every communicating rank pair
(NCCL FIFO safety).
Parity: ``resihp/runtime/hetero_runtime.py:33-148`` (same iteration steps and channel groups).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..comm.comm_manager import GenerationComms, ResilientCommManager
from ..comm.group_spec import GroupSpec
from ..comm.p2p import P2PEngine, boundary_routes, channel_name
from ..plan.hetero_plan import HeteroParallelPlan
from ..plan.ir import Op, Schedule
from ..state.rng_data import IndexAddressableSampler
from .hetero_grad_sync import HeteroGradSync, ParamShard
from .interpreter import Interpreter, RefStageExecutor
from .reference_model import ChunkedStage, RefModelConfig, RefStage, TPContext, global_tokens
from .weight_grad_store import AutogradWeightGradStore


def reference_shards(cfg: RefModelConfig, stage_module) -> dict[str, ParamShard]:
    """Partition metadata of every parameter of a reference-model stage."""
    length = {"ln": cfg.hidden, "fc1": cfg.ffn, "fc2.weight": cfg.ffn, "fc2.bias": cfg.hidden}

    def full_size(name: str) -> int:
        return length[name] if name in length else length[name.split(".")[0]]

    shards = {}
    for key in stage_module.named_state():
        name = key.split(".", 2)[2]
        shards[key] = ParamShard(key, RefStage.param_dim(key), full_size(name), stage_module.sp_partial(key))
    return shards


def reference_partition_sizes(cfg: RefModelConfig) -> tuple[int, ...]:
    return tuple(sorted({cfg.hidden, cfg.ffn}))


def channel_specs(plan: HeteroParallelPlan, schedule: Schedule, n_rows_max: int, row_counts=None) -> list[GroupSpec]:
    """2-rank groups for every (source, destination) pair a pipeline message can take.  Routes
    depend on the row count, so the union over every count a micro-batch can have is created
    (``row_counts``, default ``1..n_rows_max``)."""
    counts = list(row_counts) if row_counts is not None else list(range(1, n_rows_max + 1))
    pairs = set()
    for key, stream in schedule.items():
        src = plan.group(*key)
        for ins in (i for i in stream if i.op in (Op.SEND_ACT, Op.SEND_GRAD)):
            dst = plan.group(*ins.peer)
            for c in range(src.cp):
                pairs.update((r.src, r.dst) for n in counts
                             for r in boundary_routes(plan.slice_ranks(src, c), plan.slice_ranks(dst, c), n))
    return [GroupSpec(channel_name(a, b), (min(a, b), max(a, b)), "p2p") for a, b in sorted(pairs)]


def channel_map(comms: GenerationComms) -> dict[tuple[int, int], object]:
    """``(src rank, dst rank) -> group`` of this rank's point-to-point channels."""
    channels = {}
    for name in (n for n in comms.specs if n.startswith("p2p/") and comms.is_member(n)):
        src, dst = map(int, name.removeprefix("p2p/").split(">"))
        channels[(src, dst)] = comms.group(name)
    return channels


class HeteroRuntime:
    def __init__(self, cfg: RefModelConfig, sampler: IndexAddressableSampler, plan: HeteroParallelPlan,
                 schedule: Schedule, comms: GenerationComms, mgr: ResilientCommManager, module, *,
                 use_channels: bool = False, progress=None, hook=None, timeout: float = 120.0,
                 weight_grad_store=None, timer=None, reporter=None):
        self.cfg, self.sampler, self.plan, self.comms, self.mgr, self.module = cfg, sampler, plan, comms, mgr, module
        self.timeout, self.timer, self.reporter = timeout, timer, reporter
        me = comms.world[comms.rank]
        self.group = g = plan.group_of_device(me)
        self.replica, self.stage = g.replica, g.stage
        self.tp_group = comms.group(plan.tp_name(g, me)) if g.tp > 1 else None
        stream = schedule[(g.replica, g.stage)]
        if weight_grad_store is None and any(ins.op == Op.W for ins in stream):
            weight_grad_store = AutogradWeightGradStore(lambda: list(module.parameters()))
        self.executor = RefStageExecutor(cfg, sampler, module, plan, g.replica, g.stage, comms.rank,
                                         weight_grad_store=weight_grad_store, timer=timer)
        p2p = P2PEngine(comms.rank, mgr, channels=channel_map(comms) if use_channels else None, timeout=timeout,
                        device=cfg.device)
        self.interp = Interpreter(plan, stream, self.executor, p2p, g.replica, g.stage, (cfg.hidden,), cfg.dtype,
                                  tp_group=self.tp_group, progress=progress, hook=hook)
        self.params = module.named_state()
        self.syncs = [HeteroGradSync(plan, comms, mgr, s, g.replica, chunk.named_state(), reference_shards(cfg, chunk),
                                     tp_group=self.tp_group, timeout=timeout)
                      for s, chunk in self.executor.modules.items()]
        self.local_layers = sum(chunk.end - chunk.start for chunk in self.executor.modules.values())

    def _wait(self, work, what: str) -> None:
        self.mgr.guarded_wait(work, timeout=self.timeout, what=what)

    def _loss_share(self) -> float:
        """This rank's part of the iteration's summed loss (0 unless it runs the last stage;
        without SP every TP rank of the last stage computed the full loss, so each takes 1/tp)."""
        if self.plan.num_stages - 1 not in self.executor.modules:
            return 0.0
        share = self.executor.loss_sum
        if not (self.plan.sequence_parallel and self.group.tp > 1):
            share /= self.group.tp
        return share

    def run_iteration(self, iteration: int) -> float:
        for p in self.params.values():
            p.grad = None
        self.interp.run(iteration)
        for sync in self.syncs:
            sync.sync()
        self._finish_delayed_scaling()
        self.interp.hook(iteration, "loss")
        tokens = global_tokens(self.cfg, self.sampler, iteration)
        for p in self.params.values():
            p.grad.div_(tokens)
        loss = torch.tensor([self._loss_share()], dtype=self.cfg.dtype, device=self.cfg.device)
        self._wait(dist.all_reduce(loss, async_op=True), "loss all-reduce")
        self._report(iteration)
        return loss.item() / tokens

    def _report(self, iteration: int) -> None:
        samples = self.executor.timing_samples()
        if self.reporter is None or self.plan.ranks(self.group)[0] != self.comms.rank:
            return
        g = self.group
        self.reporter("timing", iteration=iteration, gen=self.plan.generation, devices=list(g.devices),
                      layers=self.local_layers, tp=g.tp, cp=g.cp, samples=samples)

    def _finish_delayed_scaling(self) -> None:
        """Per-layer global amax (MAX over every rank's micro-batches), then the history update;
        ranks without a layer contribute 0."""
        if not self.cfg.amax_history:
            return
        local = [b for chunk in self.executor.modules.values() for b in chunk.blocks]
        amax = torch.zeros(self.cfg.num_layers, dtype=self.cfg.dtype, device=self.cfg.device)
        for b in local:
            amax[b.layer] = b.pending_amax
        self._wait(dist.all_reduce(amax, op=dist.ReduceOp.MAX, async_op=True), "amax all-reduce")
        for b in local:
            b.finish_iteration(amax[b.layer])


def build_stage_module(cfg: RefModelConfig, plan: HeteroParallelPlan, comms: GenerationComms,
                       mgr: ResilientCommManager):
    """This device's layers: one ``RefStage``, or a ``ChunkedStage`` over its interleaved chunks."""
    me = comms.world[comms.rank]
    mine = plan.groups_of_device(me)
    g = mine[0]
    tp = TPContext(group=comms.group(plan.tp_name(g, me)) if g.tp > 1 else None,
                   rank=g.slice(g.slice_of(me)).index(me), size=g.tp, sequence_parallel=plan.sequence_parallel,
                   waiter=lambda work: mgr.guarded_wait(work, what="tp collective"))
    stages = {c.stage: RefStage(cfg, *c.layers, tp) for c in mine}
    return stages[g.stage] if len(stages) == 1 else ChunkedStage(stages)
