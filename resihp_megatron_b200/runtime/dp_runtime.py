"""Replica-level data-parallel runtime (every worker holds the whole model).

Each worker runs its assigned micro-batches and keeps a *sum* of gradients; one flat
all-reduce covers gradients plus the loss scalar, then gradients are divided by the global
token count.  ``canonical=True`` makes the result independent of the DP layout: every worker
keeps one gradient vector per micro-batch, the per-micro-batch vectors are all-gathered and
summed in global micro-batch order on every rank -- exactly the order single-process training
accumulates them -- so the loss trajectory is bit-identical before and after a
reconfiguration.  ``sync_full_state`` copies model + optimizer state from a source worker to a
lagging or new one.  (Reference: ``resihp/runtime/dp_runtime.py:14-85``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..comm.comm_manager import GenerationComms, ResilientCommManager
from ..state.rng_data import IndexAddressableSampler
from .optim import Adam


class DataParallelRuntime:
    def __init__(self, cfg, sampler: IndexAddressableSampler, model, comms: GenerationComms,
                 mgr: ResilientCommManager, assignment: list[int], *, hook=None, progress=None,
                 timeout: float = 120.0, canonical: bool = False, num_microbatches: int | None = None,
                 batch_fn=None, loss_fn=None, tokens_fn=None):
        self.cfg = cfg
        self.sampler = sampler
        self.model = model
        self.comms = comms
        self.mgr = mgr
        self.assignment = assignment
        self.hook = hook or (lambda it, phase: None)
        self.progress = progress or (lambda **kw: None)
        self.timeout = timeout
        self.canonical = canonical
        self.num_microbatches = num_microbatches or sampler.num_microbatches
        # model-specific pieces (defaults: the MLP reference model)
        if batch_fn is None:
            from .reference_model import global_tokens, microbatch, token_loss

            batch_fn = lambda it, mb: microbatch(cfg, sampler, it, mb)  # noqa: E731
            loss_fn = lambda model, m: token_loss(model(m.x), m.y, m.mask)  # noqa: E731
            tokens_fn = lambda it: global_tokens(cfg, sampler, it)  # noqa: E731
        self.batch_fn, self.loss_fn, self.tokens_fn = batch_fn, loss_fn, tokens_fn

    def _params(self):
        return list(self.model.named_state().items())

    def run_iteration(self, iteration: int) -> float:
        params = self._params()
        dtype = params[0][1].dtype
        for _, p in params:
            p.grad = None
        per_mb: dict[int, torch.Tensor] = {}
        local = 0.0
        for mb in self.assignment:
            self.hook(iteration, "forward")
            self.progress(iteration=iteration, phase=f"mb{mb}", in_collective=False)
            loss = self.loss_fn(self.model, self.batch_fn(iteration, mb))
            if self.canonical:
                grads = torch.autograd.grad(loss, [p for _, p in params], allow_unused=True)
                per_mb[mb] = torch.cat([(g if g is not None else torch.zeros_like(p)).reshape(-1)
                                        for g, (_, p) in zip(grads, params)] + [loss.detach().reshape(1)])
            else:
                loss.backward()
            local += loss.item()
        self.hook(iteration, "reduce")
        total = self.tokens_fn(iteration)
        if self.canonical:
            flat = self._canonical_reduce(per_mb, params, dtype)
        else:
            flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for _, p in params]
                             + [torch.tensor([local], dtype=dtype)])
            if self.comms.world_size > 1:
                self.progress(iteration=iteration, phase="grad_allreduce", in_collective=True)
                self.mgr.guarded_wait(dist.all_reduce(flat, async_op=True), timeout=self.timeout,
                                      what="grad all-reduce")
        off = 0
        for _, p in params:
            n = p.numel()
            p.grad = (flat[off:off + n].view_as(p) / total).clone()
            off += n
        self.hook(iteration, "step")
        return flat[-1].item() / total

    def _canonical_reduce(self, per_mb: dict[int, torch.Tensor], params, dtype) -> torch.Tensor:
        """Sum per-micro-batch vectors in global micro-batch order (layout-invariant)."""
        n = sum(p.numel() for _, p in params) + 1
        M = self.num_microbatches
        mine = torch.zeros(M, n, dtype=dtype)
        for mb, v in per_mb.items():
            mine[mb] = v
        if self.comms.world_size > 1:
            self.progress(in_collective=True, phase="grad_gather")
            # each micro-batch is computed by exactly one worker, so a SUM all-reduce of the
            # zero-padded [M, n] table reproduces every row exactly (x + 0 is exact)
            self.mgr.guarded_wait(dist.all_reduce(mine, async_op=True), timeout=self.timeout, what="grad gather")
        acc = torch.zeros(n, dtype=dtype)
        for mb in range(M):
            acc = acc + mine[mb]
        return acc


def full_state(opt: Adam, committed_iteration: int) -> tuple[dict[str, torch.Tensor], torch.Tensor]:
    return opt.state_tensors(), torch.tensor([committed_iteration, opt.step_count], dtype=torch.int64)


def sync_full_state(mgr: ResilientCommManager, comms: GenerationComms, my_id: str, sources: dict[str, str], opt: Adam,
                    committed_iteration: int, timeout: float = 120.0) -> int | None:
    """Copy model + optimizer state to each receiver from its source; returns the adopted
    iteration on receivers, ``None`` elsewhere."""
    tensors, meta = full_state(opt, committed_iteration)
    keys = sorted(tensors)
    works = []
    got = None
    rmeta = torch.zeros(2, dtype=torch.int64)
    rbuf: dict[str, torch.Tensor] = {}
    for dst, src in sorted(sources.items()):
        if my_id == src:
            peer = comms.rank_of(dst)
            works.append(dist.isend(meta, peer, tag=0))
            works.extend(dist.isend(tensors[k].contiguous(), peer, tag=i + 1) for i, k in enumerate(keys))
        if my_id == dst:
            peer = comms.rank_of(src)
            rbuf = {k: torch.empty_like(tensors[k]) for k in keys}
            works.append(dist.irecv(rmeta, peer, tag=0))
            works.extend(dist.irecv(rbuf[k], peer, tag=i + 1) for i, k in enumerate(keys))
            got = True
    for w in works:
        mgr.guarded_wait(w, timeout=timeout, what="state sync")
    if got:
        opt.load_state_tensors(rbuf, int(rmeta[1].item()))
        return int(rmeta[0].item())
    return None
