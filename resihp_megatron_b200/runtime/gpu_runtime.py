"""One generation's hybrid-parallel data plane on GPUs: TP (+ sequence parallel) x PP x DP.

Every rank runs one (replica, stage) slot of a ``HeteroParallelPlan``: a ``TPStage`` (its layer
range, its TP shard) driven by the pipeline IR ``Interpreter`` with the planner's validated
schedule; pipeline-boundary activations and gradients go over NCCL point to point (one 2-rank
channel per direction, ``comm.p2p``); tensor-parallel collectives are fused into the GEMMs over
NVLink peer memory (``tp_impl="fused"``) or run as NCCL collectives (``"collective"``, the
baseline).  After the last backward each parameter set is reduced over its data-parallel group
and updated by a sharded Adam: the tensor-parallel shards over the same TP rank of every
replica, the replicated set (norms, embedding, LM head, whose gradients are per-TP-rank partial
sums under sequence parallelism) over every rank of the stage -- the fused peer-memory step
(``dp_impl="fused"``) or reduce-scatter / Adam / all-gather (``"collective"``).

Replicas of a stage share its layer range; their TP degrees may differ (after a failure the
planner shrinks a group's TP degree): the shards are then reduced slice by slice over the holders
of each interval of the common shard refinement (``HeteroParamSync``).
(Reference: ``resihp/runtime/hetero_runtime.py:33-148`` and ``resihp/runtime/dp_runtime.py``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..comm.group_spec import GroupSpec
from ..comm.p2p import P2PEngine
from ..models.config import GPTConfig
from ..plan.hetero_plan import HeteroParallelPlan, StageGroup, dpshard_group_name, tp_group_name
from ..plan.ir import Op, Schedule
from ..utils.intervals import even_split, locate, refine
from .gpu_executor import GPUStageExecutor, TokenSource
from .hetero_runtime import channel_map, channel_specs
from .interpreter import Interpreter


def shard_group_name(stage: int, tp_rank: int) -> str:
    return f"dp/s{stage}/t{tp_rank}"


def replicated_group_name(stage: int) -> str:
    return f"dprep/s{stage}"


def stage_is_homogeneous(plan: HeteroParallelPlan, stage: int) -> bool:
    """Every replica of the stage has the same TP degree (so shard layouts coincide)."""
    return len({g.tp for g in plan.groups_at(stage)}) == 1


def check_supported(plan: HeteroParallelPlan) -> None:
    for s in range(plan.num_stages):
        gs = plan.groups_at(s)
        if len({g.layers for g in gs}) != 1:
            raise NotImplementedError(f"stage {s}: replicas hold different layer ranges")
        for g in gs:
            if g.cp != 1:
                raise NotImplementedError("context parallelism is not wired into the GPU runtime")
            r = plan.ranks(g)
            if list(r) != sorted(r):
                raise NotImplementedError(f"group r{g.replica}/s{g.stage}: devices must be in rank order")


def gpu_group_specs(plan: HeteroParallelPlan, schedule: Schedule, tokens_per_microbatch: int,
                    partitions: tuple[int, ...] = ()) -> list[GroupSpec]:
    """TP groups; per stage the data-parallel group of the replicated set and, for the
    tensor-parallel shards, one group per TP rank (replicas with equal TP degrees) or one group
    per holder set of the common shard refinement (``partitions``: the lengths of the
    tensor-parallel dimensions; replicas with different TP degrees); one channel per direction
    of every pipeline-boundary rank pair."""
    check_supported(plan)
    specs: dict[str, GroupSpec] = {}
    for g in plan.stage_groups:
        if g.tp > 1:
            n = tp_group_name(g.replica, g.stage)
            specs[n] = GroupSpec(n, plan.ranks(g), "tp")
    for s in range(plan.num_stages):
        gs = plan.groups_at(s)
        if stage_is_homogeneous(plan, s):
            for j in range(gs[0].tp):
                n = shard_group_name(s, j)
                specs[n] = GroupSpec(n, tuple(sorted(plan.ranks(g)[j] for g in gs)), "dp")
        else:
            if not partitions:
                raise ValueError("a stage with unequal TP degrees needs the partitioned dimension lengths")
            for holders in plan.dpshard_holder_sets(s, partitions):
                n = dpshard_group_name(s, holders)
                specs[n] = GroupSpec(n, holders, "dpshard")
        n = replicated_group_name(s)
        specs[n] = GroupSpec(n, tuple(sorted(r for g in gs for r in plan.ranks(g))), "dp")
    out = list(specs.values())
    out += channel_specs(plan, schedule, tokens_per_microbatch, row_counts=[tokens_per_microbatch])
    return out


class ParamSetSync:
    """Reduction over the data-parallel group + sharded Adam + weight gather of one flat
    parameter set (``FlatParams``)."""

    def __init__(self, ranks: tuple[int, ...], me: int, group, impl: str, device, *, abort=None,
                 budget_s: float = 60.0, waiter=None, zero: bool = True):
        """``zero=False`` keeps the whole optimizer state on every rank of the group (gradients
        all-reduced, every rank updates everything): redundant state that survives the loss of
        any one replica, at 12 more bytes per parameter (collective path only)."""
        self.size, self.index = len(ranks), ranks.index(me)
        self.group = group
        self.device = torch.device(device)
        self.impl = "single" if self.size == 1 else impl
        if self.impl not in ("single", "fused", "collective"):
            raise ValueError(impl)
        self.zero = zero and self.size > 1
        if not self.zero and self.impl == "fused":
            raise ValueError("the fused data-parallel step shards the optimizer state (zero=True)")
        self.wait = waiter or (lambda work: work.wait())
        self.fdp = None
        if self.impl == "fused":
            from ..parallel.dp_fused import FusedDataParallel
            from ..parallel.symm import exchange_via_group

            self.fdp = FusedDataParallel(self.index, self.size, exchange_via_group(group), self.device, abort=abort,
                                         barrier_budget_s=budget_s, spare_bank=False)
        self.P = None
        self.grad_shard = None

    @property
    def shard(self) -> tuple[int, int]:
        return (self.index, self.size) if self.zero else (0, 1)

    @property
    def factories(self):
        return (self.fdp.buffer_factory, self.fdp.opt_factory) if self.fdp is not None else (None, None)

    def attach(self, P) -> None:
        self.P = P
        if self.impl == "collective" and self.zero:
            self.grad_shard = torch.empty(P.shard_numel, dtype=torch.float32, device=self.device)

    def reduce(self) -> None:
        """The gradient reduction of the step (nothing for the fused path, which reduces inside
        ``apply``): an all-reduce (whole optimizer state) or a reduce-scatter into this rank's
        gradient shard (ZeRO-1)."""
        P = self.P
        if self.impl in ("single", "fused"):
            return
        if not self.zero:
            self.wait(dist.all_reduce(P.grad, group=self.group, async_op=True))
            return
        self.wait(dist.reduce_scatter_tensor(self.grad_shard, P.grad, group=self.group, async_op=True))
        P.grad.zero_()

    def apply(self, *, lr: float, betas, eps: float, weight_decay: float) -> None:
        """Adam on this rank's optimizer state (after ``reduce``) and the weight gather."""
        P = self.P
        P.step += 1
        if self.impl == "fused":
            self.fdp.step(P, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
            return
        kw = dict(lr=lr, beta1=betas[0], beta2=betas[1], eps=eps, weight_decay=weight_decay, step=P.step)
        if self.impl == "single" or not self.zero:
            ops.adam_step(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.bf16, zero_grad=True, **kw)
            return
        mine = P.shard_slice(P.bf16)
        ops.adam_step(P.master, self.grad_shard, P.exp_avg, P.exp_avg_sq, mine, zero_grad=False, **kw)
        src = mine if dist.get_backend(self.group) == "nccl" else mine.clone()
        self.wait(dist.all_gather_into_tensor(P.bf16, src, group=self.group, async_op=True))

    def step(self, **kw) -> None:
        self.reduce()
        self.apply(**kw)

    def discard(self) -> None:
        """Drop this step's gradients (an aborted iteration)."""
        self.P.grad.zero_()

    def check(self) -> None:
        if self.fdp is not None:
            self.fdp.check()

    def close(self) -> None:
        if self.fdp is not None:
            self.fdp.close()
            self.fdp = None


class HeteroParamSync:
    """Data-parallel reduction of the tensor-parallel shards when the replicas of a stage use
    different TP degrees.  On the common refinement of every replica's shard boundaries each
    interval has exactly one holder per replica; those holders all-reduce exactly that slice
    (all slices of one holder set packed into one flat buffer, one all-reduce per set), then
    every rank applies Adam to its whole local shard (optimizer state not sharded: local
    layouts differ across the group).  (Reference: ``resihp/runtime/hetero_grad_sync.py:60-120``.)"""

    impl = "hetero"
    shard = (0, 1)
    factories = (None, None)
    size, group = 1, None

    def __init__(self, plan: HeteroParallelPlan, stage: int, me: int, comms, device, waiter=None):
        self.plan, self.stage, self.me, self.comms = plan, stage, me, comms
        self.device = torch.device(device)
        self.wait = waiter or (lambda work: work.wait())
        self.P = None
        self.slices: dict[tuple[int, ...], list[tuple[str, int, int, int]]] = {}

    def attach(self, P) -> None:
        self.P = P
        tp_slices = self.plan.tp_slices(self.stage)
        for name in P.order:
            s = P.specs[name]
            if s.shard_dim is None:
                continue
            n = s.full_shape[s.shard_dim]
            parts = [even_split(n, len(sl)) for sl in tp_slices]
            for iv in refine(parts):
                holders = tuple(sorted(self.plan.rank(sl[locate(part, iv)]) for sl, part in zip(tp_slices, parts)))
                if self.me not in holders or len(holders) == 1:
                    continue
                self.slices.setdefault(holders, []).append((name, s.shard_dim, iv[0] - s.shard_range[0],
                                                            iv[1] - iv[0]))

    def reduce(self) -> None:
        P = self.P
        for holders, pieces in self.slices.items():
            views = [P.g(name).narrow(dim, lo, ln) for name, dim, lo, ln in pieces]
            flat = torch.cat([v.reshape(-1) for v in views])
            self.wait(dist.all_reduce(flat, group=self.comms.group(dpshard_group_name(self.stage, holders)),
                                      async_op=True))
            off = 0
            for v in views:
                v.copy_(flat[off:off + v.numel()].view(v.shape))
                off += v.numel()

    def apply(self, *, lr: float, betas, eps: float, weight_decay: float) -> None:
        P = self.P
        P.step += 1
        ops.adam_step(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.bf16, lr=lr, beta1=betas[0], beta2=betas[1],
                      eps=eps, weight_decay=weight_decay, step=P.step, zero_grad=True)

    def step(self, **kw) -> None:
        self.reduce()
        self.apply(**kw)

    def discard(self) -> None:
        self.P.grad.zero_()

    def check(self) -> None:
        pass

    def close(self) -> None:
        pass


class HeteroFusedSync(HeteroParamSync):
    """``HeteroParamSync`` on NVLink peer memory: every rank packs its slices of each holder set
    into its own region of a symmetric heap (one strided-copy launch), and after a bounded barrier
    sums every slice of its sets from all holders' regions in rank order (one launch; every holder
    computes the same bits), unpacks the sums into its gradient (one launch) and passes a second
    barrier before its region may be rewritten.  The piece tables are built once and stay on the
    device.  Region offsets of every rank follow from the plan (each rank's sets in sorted order),
    so no layout is exchanged.  Falls back to the library path when a slice is not 16-byte aligned
    or a set has more than 8 holders.  (Reference: the same reduction with one all-reduce per
    holder set, ``resihp/runtime/hetero_grad_sync.py:60-120``.)"""

    impl = "hetero-fused"

    def __init__(self, plan: HeteroParallelPlan, stage: int, me: int, comms, device, *, exchange=None, abort=None,
                 budget_s: float = 60.0, waiter=None, _heap=None, _ranks=None):
        super().__init__(plan, stage, me, comms, device, waiter)
        self.exchange, self.abort, self.budget = exchange, abort, budget_s
        self.ranks = _ranks or tuple(sorted(r for g in plan.groups_at(stage) for r in plan.ranks(g)))
        self._heap_in = _heap
        self.heap = None
        self.fused = False

    def _all_sets(self, P) -> dict[tuple[int, ...], list[tuple[str, int, int]]]:
        """Every holder set of the stage with its pieces ``(name, global interval start, length)``."""
        tp_slices = self.plan.tp_slices(self.stage)
        out: dict[tuple[int, ...], list[tuple[str, int, int]]] = {}
        for name in P.order:
            sp = P.specs[name]
            if sp.shard_dim is None:
                continue
            n = sp.full_shape[sp.shard_dim]
            parts = [even_split(n, len(sl)) for sl in tp_slices]
            for iv in refine(parts):
                holders = tuple(sorted(self.plan.rank(sl[locate(part, iv)]) for sl, part in zip(tp_slices, parts)))
                if len(holders) > 1:
                    out.setdefault(holders, []).append((name, iv[0], iv[1] - iv[0]))
        return out

    def attach(self, P) -> None:
        super().attach(P)
        sets, size, offsets, totals, geo = self.layout(P)
        self._build(P, sets, size, offsets, totals, geo)

    def layout(self, P):
        """``(sets, size, offsets, totals, geo)``: every holder set of the stage with its pieces,
        each set's element count, every rank's region offset of each of its sets (elements), every
        rank's region total, and this rank's pieces ``(set, offset in the set's region, grad
        pointer, rows, row bytes, row pitch)`` -- pure index arithmetic from the plan and specs."""
        sets = self._all_sets(P)

        def piece_numel(name: str, ln: int) -> int:
            sp = P.specs[name]
            other = 1
            for d, v in enumerate(sp.full_shape):
                if d != sp.shard_dim:
                    other *= v
            return ln * other

        size = {h: sum(piece_numel(nm, ln) for nm, _, ln in pcs) for h, pcs in sets.items()}
        offsets: dict[int, dict[tuple[int, ...], int]] = {}
        totals = {}
        for r in self.ranks:
            off = 0
            offsets[r] = {}
            for h in sorted(sets):
                if r in h:
                    offsets[r][h] = off
                    off += (size[h] + 3) // 4 * 4  # 16-byte aligned regions
            totals[r] = off
        mine = sorted(self.slices)
        # piece geometry of this rank's slices: (grad pointer offset bytes, rows, row bytes, pitch bytes)
        geo = []
        for h in mine:
            poff = 0
            for name, dim, lo, ln in self.slices[h]:
                g = P.g(name)
                if dim == 0:
                    row = g[0].numel() if g.dim() > 1 else 1
                    item = (g.data_ptr() + lo * row * 4, 1, ln * row * 4, ln * row * 4)
                else:
                    item = (g.data_ptr() + lo * 4, g.shape[0], ln * 4, g.shape[1] * 4)
                geo.append((h, poff, *item))
                poff += piece_numel(name, ln)
        return sets, size, offsets, totals, geo

    def _build(self, P, sets, size, offsets, totals, geo) -> None:
        mine = sorted(self.slices)
        ok = bool(mine) and all(len(h) <= 8 for h in mine)
        ok = ok and not any((a | c | d) & 15 for _, _, a, _, c, d in geo) and not any(o & 3 for _, o, *_ in geo)
        if self.comms is not None:  # every rank of the stage takes the same path (the heap is collective)
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
            self.wait(dist.all_reduce(flag, op=dist.ReduceOp.MIN,
                                      group=self.comms.group(replicated_group_name(self.stage)), async_op=True))
            ok = bool(flag.item())
        if not ok:
            return  # a slice that is not 16-byte aligned or a set of more than 8 holders: library path
        from ..parallel.symm import SymmetricHeap

        cap = max(max(totals.values()), 64)
        idx = self.ranks.index(self.me)
        self.heap = self._heap_in or SymmetricHeap({"region": (cap, torch.float32)}, idx, len(self.ranks),
                                                   self.exchange, self.device, self.abort)
        base = self.heap.peer_ptrs("region")
        self.scratch = torch.empty(max(totals[self.me], 4), dtype=torch.float32, device=self.device)
        pack, unpack = [], []
        for h, poff, src, rows, row_bytes, pitch in geo:
            dst = base[idx] + (offsets[self.me][h] + poff) * 4
            scr = self.scratch.data_ptr() + (offsets[self.me][h] + poff) * 4
            pack += [src, dst, rows, row_bytes, pitch, row_bytes]
            unpack += [scr, src, rows, row_bytes, row_bytes, pitch]
        sums = []
        for h in mine:
            srcs = [base[self.ranks.index(r)] + offsets[r][h] * 4 for r in h]
            sums += [self.scratch.data_ptr() + offsets[self.me][h] * 4, size[h], len(h)] + srcs + [0] * (8 - len(h))
        dev = self.device.index if self.device.index is not None else 0
        from ..ops._build import ext

        self.pack_t, self.pack_n = ext().symm_copy2d_build(pack, dev)
        self.unpack_t, self.unpack_n = ext().symm_copy2d_build(unpack, dev)
        self.sum_t, self.sum_n = ext().symm_sum_build(sums, dev)
        self.fused = True

    # the three phases (emulated ranks in one process call them in turn, without barriers)
    def pack(self) -> None:
        from ..ops._build import ext

        ext().symm_copy2d_run(self.pack_t, self.pack_n)
        ops.count(1)

    def sum(self) -> None:
        from ..ops._build import ext

        ext().symm_sum_run(self.sum_t, self.sum_n)
        ops.count(1)

    def unpack(self) -> None:
        from ..ops._build import ext

        ext().symm_copy2d_run(self.unpack_t, self.unpack_n)
        ops.count(1)

    def reduce(self) -> None:
        if not self.fused:
            return super().reduce()
        self.pack()
        self.heap.barrier(self.budget)  # every holder's slices are in its region
        self.sum()
        self.heap.barrier(self.budget)  # every region has been read: it may be rewritten next step
        self.unpack()
        ops.count(2)

    def check(self) -> None:
        if self.heap is not None and self._heap_in is None:
            self.heap.check()

    def close(self) -> None:
        if self.heap is not None and self._heap_in is None:
            self.heap.close()
        self.heap = None

    def close(self) -> None:
        pass


class GPUHybridRuntime:
    def __init__(self, cfg: GPTConfig, plan: HeteroParallelPlan, schedule: Schedule, comms, mgr, *, device,
                 micro_batch: int = 1, seq_len: int | None = None, tokens: TokenSource | None = None,
                 tp_impl: str = "fused", dp_impl: str = "fused", seed: int = 0, lr: float = 3e-4,
                 betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0, budget_s: float = 60.0,
                 progress=None, hook=None, zero: bool = True, init: bool = True, fp8=None):
        """``zero``: shard the optimizer state over each data-parallel group (ZeRO-1) or keep it
        whole on every replica (redundant: survives a fail-stop); ``init``: draw the initial
        weights (False when a migrated state is loaded next); ``fp8``: an ``Fp8Recipe`` --
        block-scaled fp8 projections whose per-layer amax is reduced with MAX over every rank at
        the end of each iteration (one all-reduce) and pushed into the amax history."""
        from ..models.tp_stage import TPStage

        check_supported(plan)
        self.cfg, self.plan, self.comms, self.mgr = cfg, plan, comms, mgr
        self.device = torch.device(device)
        self.S = seq_len or cfg.seq_len
        self.micro_batch = micro_batch
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        me = comms.world[comms.rank]
        g: StageGroup = plan.group_of_device(me)
        if g is None:
            raise RuntimeError(f"{me} has no slot in generation {plan.generation} (standby)")
        self.group, self.replica = g, g.replica
        ranks = plan.ranks(g)
        tp_rank = ranks.index(comms.rank)
        T = micro_batch * self.S
        self.tokens_per_step = plan.num_microbatches * T
        waiter = (lambda w: mgr.guarded_wait(w, what="data-parallel collective")) if mgr is not None else None
        self.abort = None
        if "fused" in (tp_impl, dp_impl):
            from ..parallel.symm import AbortWord

            self.abort = AbortWord()
            if mgr is not None:
                mgr.add_abort_hook(self.abort.set)
        # tensor parallelism
        tp_pg = comms.group(tp_group_name(g.replica, g.stage)) if g.tp > 1 else None
        from ..parallel import tp_backend

        self.sp = plan.sequence_parallel or g.tp == 1
        if g.tp == 1:
            self.tp = tp_backend.SoloTP(self.device)
        elif tp_impl == "fused":
            from ..parallel.symm import exchange_via_group
            from ..parallel.tp_fused import TensorParallelComm

            comm = TensorParallelComm(tp_rank, g.tp, exchange_via_group(tp_pg), self.device, max_rows=T,
                                      max_k=cfg.hidden, max_n=cfg.hidden, abort=self.abort, budget_s=budget_s)
            self.tp = tp_backend.FusedTP(comm, sp=self.sp)
        elif tp_impl == "collective":
            self.tp = tp_backend.CollectiveTP(tp_rank, g.tp, tp_pg, self.device,
                                              waiter=(lambda w: mgr.guarded_wait(w, what="tp collective"))
                                              if mgr is not None else None, sp=self.sp)
        else:
            raise ValueError(tp_impl)
        # one model chunk per virtual stage this device runs (one without interleaving); data
        # parallelism per chunk: the sharded set over the same TP rank of every replica, the
        # replicated set over the whole stage
        self.chunks: dict[int, tuple] = {}
        for c in plan.groups_of_device(me):
            stage_groups = plan.groups_at(c.stage)
            rep_ranks = tuple(sorted(r for h in stage_groups for r in plan.ranks(h)))
            if stage_is_homogeneous(plan, c.stage):
                shd_ranks = tuple(sorted(plan.ranks(h)[tp_rank] for h in stage_groups))
                shd_sync = ParamSetSync(shd_ranks, comms.rank, comms.group(shard_group_name(c.stage, tp_rank)), dp_impl,
                                        self.device, abort=self.abort, budget_s=budget_s, waiter=waiter, zero=zero)
            elif dp_impl == "fused" and self.device.type == "cuda":
                from ..parallel.symm import exchange_via_group

                shd_sync = HeteroFusedSync(plan, c.stage, comms.rank, comms, self.device,
                                           exchange=exchange_via_group(comms.group(replicated_group_name(c.stage))),
                                           abort=self.abort, budget_s=budget_s, waiter=waiter)
            else:
                shd_sync = HeteroParamSync(plan, c.stage, comms.rank, comms, self.device, waiter=waiter)
            rep_sync = ParamSetSync(rep_ranks, comms.rank, comms.group(replicated_group_name(c.stage)), dp_impl,
                                    self.device, abort=self.abort, budget_s=budget_s, waiter=waiter, zero=zero)
            stage = TPStage(cfg, self.device, layers=range(*c.layers), first=c.stage == 0,
                            last=c.stage == plan.num_stages - 1, tp=self.tp, micro_batch=micro_batch, seq_len=self.S,
                            seed=seed, rep_shard=rep_sync.shard, shd_shard=shd_sync.shard,
                            rep_factories=rep_sync.factories, shd_factories=shd_sync.factories, init=init,
                            fp8=fp8, sp=self.sp)
            rep_sync.attach(stage.rep)
            shd_sync.attach(stage.shd)
            self.chunks[c.stage] = (stage, rep_sync, shd_sync)
        self.tokens = tokens or TokenSource(cfg.vocab_size, micro_batch, self.S)
        self.executor = GPUStageExecutor({s_: ch[0] for s_, ch in self.chunks.items()}, plan, g.replica, comms.rank,
                                         self.tokens, grad_scale=1.0 / self.tokens_per_step, sp=self.sp)
        stream = schedule[(g.replica, g.stage)]
        self.executor.split_backward = any(ins.op == Op.W for ins in stream)
        p2p = P2PEngine(comms.rank, mgr, channels=channel_map(comms), device=str(self.device))
        self.interp = Interpreter(plan, stream, self.executor, p2p, g.replica, g.stage, (cfg.hidden,), torch.bfloat16,
                                  tp_group=tp_pg, progress=progress, hook=hook)
        self.iteration = 0
        self.hook = hook
        self.fp8 = fp8
        self._amax = None
        if fp8 is not None:
            from ..models.fp8_linear import NSLOTS

            self._amax = torch.zeros(cfg.layers, NSLOTS, dtype=torch.float32, device=self.device)

    # ------------------------------------------------------------------ chunk views
    @property
    def stage(self):
        """The model chunk (a device runs one unless the plan interleaves stages)."""
        if len(self.chunks) != 1:
            raise AttributeError("interleaved plan: use .chunks")
        return next(iter(self.chunks.values()))[0]

    def _syncs(self):
        for _, rep_sync, shd_sync in self.chunks.values():
            yield shd_sync
            yield rep_sync

    def param_sets(self) -> list[tuple]:
        """``(FlatParams, sync)`` of every parameter set of every chunk."""
        out = []
        for stage, rep_sync, shd_sync in self.chunks.values():
            out += [(stage.rep, rep_sync), (stage.shd, shd_sync)]
        return out

    @property
    def step_count(self) -> int:
        return next(iter(self.chunks.values()))[0].shd.step

    def inflight(self) -> int:
        return sum(ch[0].inflight() for ch in self.chunks.values())

    def buffers(self) -> dict[str, torch.Tensor]:
        """Non-trainable state an iteration mutates, by logical key (the fp8 amax histories of
        this rank's layers): migrated with its layer, rolled back with an aborted iteration."""
        out = {}
        for stage, _, _ in self.chunks.values():
            if stage.f8 is not None:
                out.update(stage.f8.state())
        return out

    def _finish_fp8(self) -> None:
        """Global per-layer amax (MAX over every rank's micro-batches and shards: one
        all-reduce over the world for all layers), then each layer's history update.
        (Reference: ``resihp/runtime/hetero_runtime.py:122-134``.)"""
        stages = [ch[0] for ch in self.chunks.values() if ch[0].f8 is not None]
        self._amax.zero_()
        for st in stages:
            self._amax[st.layer_ids] = st.f8.pending
        # MAX over the bit patterns (non-negative floats order like ints; NaN stays the largest)
        work = dist.all_reduce(self._amax.view(torch.int32), op=dist.ReduceOp.MAX, async_op=True)
        if self.mgr is not None:
            self.mgr.guarded_wait(work, what="amax all-reduce")
        else:
            work.wait()
        for st in stages:
            st.f8.pending.copy_(self._amax[st.layer_ids])
            st.f8.finish_iteration()

    def fp8_nonfinite(self) -> bool:
        """Whether the iteration's reduced amax of any layer of this rank is inf / NaN."""
        return any(ch[0].f8.has_nonfinite() for ch in self.chunks.values() if ch[0].f8 is not None)

    def after_backward(self, iteration: int) -> None:
        """Between the last backward of an iteration and the gradient reduction: the replicated
        set's gradient share under plain TP, the fp8 amax reduction and history update, the
        ``loss`` hook."""
        if not self.sp:
            # plain TP: every rank of a replica computed the replicated parameters' full gradient;
            # the replicated set is reduced over all ranks of the stage, so each counts 1 / tp
            for stage, _, _ in self.chunks.values():
                stage.rep.grad.mul_(1.0 / self.group.tp)
        if self.fp8 is not None:
            self._finish_fp8()
        if self.hook is not None:  # after the loss and the amax reduction, before the gradient reduction
            self.hook(iteration, "loss")

    def run_iteration(self, iteration: int | None = None, step: bool = True) -> torch.Tensor:
        """One training step of this slot; returns the global mean token loss as a 0-d device
        tensor (no host synchronisation).  ``step=False`` stops after the gradient reduction
        (the resilient loop applies the optimizer step once the iteration is REDUCED)."""
        it = self.iteration if iteration is None else iteration
        self.interp.run(it)
        self.after_backward(it)
        if self.fp8 is not None and self.fp8.skip_nonfinite and self.fp8_nonfinite():
            # every rank sees the same reduced amax, so every rank drops the iteration
            self.discard_grads()
            self.skipped_steps = getattr(self, "skipped_steps", 0) + 1
            step = None
        else:
            for sync in self._syncs():
                sync.reduce()
        if step:
            self.apply_step()
        # the loss travels with a count of the ranks that took part: an NCCL collective cut short
        # by a dead peer or an abort looks complete to the host, but its count falls short
        loss_and_count = torch.stack([self.executor.loss_sum.reshape(()).float(),
                                      torch.ones((), dtype=torch.float32, device=self.device)])
        work = dist.all_reduce(loss_and_count, async_op=True)
        if self.mgr is not None:
            self.mgr.guarded_wait(work, what="loss all-reduce")
        else:
            work.wait()
        self.iteration = it + 1
        self.last_participants = loss_and_count[1]
        return loss_and_count[0] / self.tokens_per_step

    def apply_step(self) -> None:
        kw = dict(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.wd)
        for sync in self._syncs():
            sync.apply(**kw)

    def discard_grads(self) -> None:
        for sync in self._syncs():
            sync.discard()

    def check(self) -> None:
        """Raise if a peer barrier of a fused collective timed out or was aborted."""
        for s in self._syncs():
            s.check()
        if hasattr(self.tp, "check"):
            self.tp.check()

    def close(self) -> None:
        """Release the symmetric heaps (before the process groups are destroyed)."""
        if torch.cuda.is_available() and self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        for s in self._syncs():
            s.close()
        self.tp.close()
        if self.abort is not None:
            self.abort.close()
            self.abort = None
