"""GPU training engine: one process per GPU, data parallel with a sharded optimizer (ZeRO-1).

``GPUTrainer.train_step(ids, labels)`` is the public entry point: it takes one step's token
ids and labels for this rank (pinned host tensors), copies them to the device, runs every
micro-batch forward and backward on the package's kernels, reduces the gradients across the
data-parallel group, applies Adam to this rank's shard of the fp32 master weights, gathers
the updated bf16 weights, and returns the step's mean token loss.  With ``dp_impl="fused"``
(default) reduction, Adam and gather are one kernel over NVLink peer memory
(``parallel.dp_fused``); ``"nccl"`` uses reduce-scatter / Adam / all-gather.

Gradients are scaled by ``1 / tokens in the global batch`` inside the cross-entropy kernel,
so the reduced gradient is the gradient of the global mean loss whatever the DP degree.
The global batch and the order of micro-batches are those of the failure-free run: rank r of
a DP group of size d takes sequences ``[r * B / d, (r + 1) * B / d)`` of every global batch
(the reference keeps the same invariant with its index-addressable sampler,
``resihp/state/rng_data.py:41``).
"""

from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist

from ..models.config import GPTConfig
from ..models.gpt import LlamaModel


class GPUTrainer:
    def __init__(self, cfg: GPTConfig, *, global_batch: int, micro_batch: int = 1, seq_len: int | None = None,
                 lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0, seed: int = 0,
                 device=None, dp_group: dist.ProcessGroup | None = None, dp_impl: str = "fused",
                 spare_bank: bool | None = None, fp8=None):
        """``fp8``: an ``Fp8Recipe`` -- block-scaled fp8 linear layers whose per-layer amax is
        reduced with MAX over the data-parallel group and recorded in the amax history at the
        end of every step."""
        self.cfg = cfg
        self.S = seq_len or cfg.seq_len
        self.group = dp_group
        self.dp = dist.get_world_size(dp_group) if (dist.is_initialized() and dp_group is not None) else 1
        self.rank = dist.get_rank(dp_group) if self.dp > 1 else 0
        if global_batch % self.dp:
            raise ValueError(f"global batch {global_batch} is not divisible by DP={self.dp}")
        self.global_batch = global_batch
        self.local_batch = global_batch // self.dp
        if self.local_batch % micro_batch:
            raise ValueError("local batch must be a multiple of the micro-batch")
        self.micro_batch = micro_batch
        self.n_micro = self.local_batch // micro_batch
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.device = torch.device(device if device is not None else f"cuda:{torch.cuda.current_device()}")
        if dp_impl not in ("fused", "nccl"):
            raise ValueError(dp_impl)
        self.dp_impl = dp_impl if self.dp > 1 else "single"
        self.fused = None
        factory = opt_factory = None
        if self.dp_impl == "fused":
            from ..parallel.dp_fused import FusedDataParallel
            from ..parallel.symm import AbortWord, exchange_via_group

            from ..models.gpt import model_param_specs
            from ..models.params import ALIGN, FlatParams

            self.abort_word = AbortWord()
            cap = FlatParams.flat_numel(model_param_specs(cfg, list(range(cfg.layers)), True, True), 1) + ALIGN * self.dp
            self.fused = FusedDataParallel(self.rank, self.dp, exchange_via_group(dp_group), self.device,
                                           abort=self.abort_word, numel_cap=cap, spare_bank=spare_bank)
            factory, opt_factory = self.fused.buffer_factory, self.fused.opt_factory
        self.model = LlamaModel(cfg, self.device, micro_batch=micro_batch, seq_len=self.S, seed=seed,
                                shard_rank=self.rank, shard_count=self.dp, buffer_factory=factory,
                                opt_factory=opt_factory, fp8=fp8)
        self.tokens_per_step = global_batch * self.S
        self.batch_offset = self.rank * self.local_batch  # first sequence of this rank in the global batch
        self.ids_dev = torch.empty(self.local_batch, self.S, dtype=torch.int64, device=self.device)
        self.labels_dev = torch.empty_like(self.ids_dev)
        P = self.model.params
        if self.dp_impl == "nccl":
            self.grad_shard = torch.empty(P.shard_numel, dtype=torch.float32, device=self.device)
        self.step_count = 0

    # ------------------------------------------------------------------ CUDA graphs
    def capture_graphs(self) -> None:
        """Capture one whole device step -- every micro-batch's forward and backward and the
        optimizer update -- into a CUDA graph; ``step_device`` then replays it (one launch from
        the host per step instead of thousands).  Single GPU only (no collective in the step).
        Call it after at least one eager step (allocator pools and kernel attributes settle)."""
        if self.dp != 1:
            raise NotImplementedError("graph capture of the data-parallel step (collectives) is not wired")
        from .. import ops

        self.drop_graphs()
        self.bias_corr = torch.zeros(2, dtype=torch.float32, device=self.device)
        # pinned staging ring: a slot is rewritten only after its previous copy ran (event), so the
        # host can run ahead of the device without racing the asynchronous copies
        self._bc_ring = torch.zeros(64, 2, dtype=torch.float32).pin_memory()
        self._bc_events: list = [None] * 64
        if self.model.f8 is not None:
            self.model.f8.version = None  # the weight quantisation is part of every replay
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        l0 = ops.launches()
        with torch.cuda.graph(g):
            self.graph_loss = self._step_body(self.ids_dev, self.labels_dev, self.bias_corr)
        self.graph_launches = ops.launches() - l0
        self.graph = g

    def drop_graphs(self) -> None:
        self.graph = None
        self.graph_loss = None

    def _step_body(self, ids: torch.Tensor, labels: torch.Tensor, bias_corr: torch.Tensor | None) -> torch.Tensor:
        from .. import ops

        m = self.model
        m.loss_acc.zero_()
        scale = 1.0 / self.tokens_per_step
        mb = self.micro_batch
        for i in range(self.n_micro):
            m.forward_backward(ids[i * mb:(i + 1) * mb].reshape(-1), labels[i * mb:(i + 1) * mb].reshape(-1), scale)
        if m.f8 is not None:
            m.f8.finish_iteration()
        P = self.model.params
        ops.adam_step(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.bf16, lr=self.lr, beta1=self.betas[0],
                      beta2=self.betas[1], eps=self.eps, weight_decay=self.wd, step=max(P.step, 1), zero_grad=True,
                      bias_corr=bias_corr)
        return m.loss_acc / self.tokens_per_step

    def _replay(self, ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        from .. import ops

        if ids.data_ptr() != self.ids_dev.data_ptr():
            self.ids_dev.copy_(ids)
            self.labels_dev.copy_(labels)
        import math

        P = self.model.params
        P.step += 1
        k = P.step % len(self._bc_events)
        if self._bc_events[k] is not None:
            self._bc_events[k].synchronize()
        self._bc_ring[k, 0] = 1.0 - self.betas[0] ** P.step
        self._bc_ring[k, 1] = math.sqrt(1.0 - self.betas[1] ** P.step)
        self.bias_corr.copy_(self._bc_ring[k], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._bc_events[k] = ev
        self.graph.replay()
        ops.count(self.graph_launches)
        self.step_count += 1
        return self.graph_loss

    # ------------------------------------------------------------------ device-resident step
    def step_device(self, ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """One optimizer step on device-resident ``[local_batch, S]`` ids/labels; returns the
        global mean loss as a 0-d device tensor (no host synchronisation)."""
        if getattr(self, "graph", None) is not None:
            return self._replay(ids, labels)
        m = self.model
        m.loss_acc.zero_()
        scale = 1.0 / self.tokens_per_step
        mb = self.micro_batch
        for i in range(self.n_micro):
            m.forward_backward(ids[i * mb:(i + 1) * mb].reshape(-1), labels[i * mb:(i + 1) * mb].reshape(-1), scale)
        if m.f8 is not None:  # the amax reduction (one MAX all-reduce) and the history update
            m.f8.finish_iteration(self._reduce_max if self.dp > 1 else None)
            if m.f8.recipe.skip_nonfinite and m.f8.has_nonfinite():  # every rank sees the same amax
                m.params.grad.zero_()
                if self.dp > 1:
                    dist.all_reduce(m.loss_acc, group=self.group)
                self.skipped_steps = getattr(self, "skipped_steps", 0) + 1
                self.step_count += 1
                return m.loss_acc / self.tokens_per_step
        self._reduce_and_update()
        self.step_count += 1
        return m.loss_acc / self.tokens_per_step

    def _reduce_max(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)

    def _reduce_and_update(self) -> None:
        from .. import ops

        P = self.model.params
        P.step += 1
        kw = dict(lr=self.lr, beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, weight_decay=self.wd,
                  step=P.step)
        if self.dp == 1:
            ops.adam_step(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.bf16, zero_grad=True, **kw)
            return
        if self.dp_impl == "fused":
            dist.all_reduce(self.model.loss_acc, group=self.group)
            self.fused.step(P, lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.wd)
            ops.count(3)  # barrier, fused step, barrier
            return
        dist.reduce_scatter_tensor(self.grad_shard, P.grad, op=dist.ReduceOp.SUM, group=self.group)
        dist.all_reduce(self.model.loss_acc, group=self.group)
        P.grad.zero_()
        ops.adam_step(P.master, self.grad_shard, P.exp_avg, P.exp_avg_sq, P.shard_slice(P.bf16), zero_grad=False,
                      **kw)
        dist.all_gather_into_tensor(P.bf16, P.shard_slice(P.bf16), group=self.group)

    # ------------------------------------------------------------------ public end-to-end step
    def train_step(self, ids_host: torch.Tensor, labels_host: torch.Tensor) -> float:
        """Copy this rank's inputs (pinned host ``[local_batch, S]`` int64) to the device, run the
        step, and return the global mean token loss read back to the host."""
        self.ids_dev.copy_(ids_host, non_blocking=True)
        self.labels_dev.copy_(labels_host, non_blocking=True)
        loss = self.step_device(self.ids_dev, self.labels_dev)
        value = float(loss.item())
        self.check()
        return value

    def check(self) -> None:
        """Raise ``PeerTimeout`` / ``PeerAborted`` if a peer barrier of the fused data-parallel
        step failed since the heap was built (synchronises with the device)."""
        if self.fused is not None:
            self.fused.check()

    # ------------------------------------------------------------------ live reconfiguration
    def shrink(self, survivors: list[int], new_group) -> bool:
        """Planned removal of data-parallel ranks with live state migration (e.g. evicting a
        fail-slow GPU).  Every current rank calls it between steps; ``survivors`` are the kept
        ranks (old numbering, ascending) and ``new_group`` their process group.  Each survivor pulls
        its new optimizer shard -- fp32 master weights and both Adam moments -- from the old owners'
        current bank into its spare bank over NVLink with one copy kernel (the departing ranks are
        sources too, so no state is lost); weights and gradients stay where they are (their layout
        does not depend on the sharding) and every peer mapping is reused; the global batch is
        re-split by largest remainder.  Returns False on a rank that leaves.  (Reference: the
        transfer engine's slice migration, ``resihp/state/transfer_engine.py:24-59``, and the DP
        planner's batch-preserving assignment, ``resihp/plan/dp_planner.py:11-22``.)"""
        import time

        from ..models.params import FlatParams
        from ..ops._build import ext
        from ..parallel.dp_fused import reshard_pull_plan
        from ..plan.dp_migration import largest_remainder

        fdp = self.fused
        if fdp is None or fdp.banks != 2:
            raise RuntimeError("live shrink needs the fused data-parallel path with a spare optimizer bank")
        marks = [("start", time.perf_counter())]

        def mark(name: str) -> None:
            torch.cuda.synchronize(self.device)
            marks.append((name, time.perf_counter()))

        old_P, heap = self.model.params, fdp.heap
        specs = self.model.param_specs
        heap.barrier(fdp.budget)  # every rank finished its last step
        torch.cuda.synchronize(self.device)
        fdp.check()
        mark("drain")
        leaving = self.rank not in survivors
        nb = 1 - fdp.bank
        moved = 0
        if not leaving:
            new_rank, new_world = survivors.index(self.rank), len(survivors)
            numel = FlatParams.flat_numel(specs, new_world)
            new_shard = numel // new_world
            dst = {k: heap.peer_ptrs(f"{k}{nb}")[self.rank] for k in fdp.STATE}
            for k in fdp.STATE:
                heap.tensor(f"{k}{nb}")[:new_shard].zero_()  # padding past the old flat size
            triples = reshard_pull_plan(self.dp, old_P.shard_numel, fdp.state_ptrs(fdp.bank), new_rank * new_shard,
                                        (new_rank + 1) * new_shard, dst, old_P.numel)
            ext().symm_copy(triples, self.device.index if self.device.index is not None else 0)
            moved = sum(triples[2::3])
        mark("migrate")
        heap.barrier(fdp.budget)  # every pull from this rank's memory has landed
        torch.cuda.synchronize(self.device)
        fdp.check()
        if leaving:
            fdp.close()
            self.fused = None
            return False
        heap.restrict(survivors)
        dist.barrier(group=new_group)  # every survivor cleared its signal pad
        mark("regroup")
        fdp.rank, fdp.world, fdp.bank = new_rank, new_world, nb
        new_P = FlatParams(specs, self.device, shard_rank=new_rank, shard_count=new_world,
                           buffer_factory=fdp.buffer_factory, opt_factory=fdp.opt_factory)
        new_P.step = self.step_count
        self.model.params = new_P
        self.group, self.rank, self.dp = new_group, new_rank, new_world
        shares = largest_remainder(self.global_batch, [1.0] * self.dp)
        self.local_batch = shares[self.rank]
        self.batch_offset = sum(shares[:self.rank])
        mb = self.micro_batch if self.local_batch % self.micro_batch == 0 else 1
        if mb != self.micro_batch:
            self.model.release_buffers()
            self.model.restore_buffers(mb)
        self.micro_batch, self.n_micro = mb, self.local_batch // mb
        self.ids_dev = torch.empty(self.local_batch, self.S, dtype=torch.int64, device=self.device)
        self.labels_dev = torch.empty_like(self.ids_dev)
        mark("commit")
        self.last_reconfig = {name: round(t - marks[i][1], 4) for i, (name, t) in enumerate(marks[1:])}
        self.last_reconfig["migrated_bytes"] = moved
        return True

    def close(self) -> None:
        """Release the symmetric heap (before the process group is destroyed)."""
        if self.fused is not None:
            self.fused.close()
            self.fused = None


def init_distributed(timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialise NCCL from torchrun's environment; returns (rank, world, local_rank)."""
    import os

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=torch.device("cuda", local))
    return rank, world, local
