"""Replica-level data-parallel runtime: every worker holds the whole model.

A worker runs the micro-batches assigned to it and keeps a *sum* of gradients; one flat
all-reduce carries the gradients and the loss, after which the gradients are divided by the
global token count.  ``canonical=True`` makes the result independent of the DP layout: each
worker keeps one gradient vector per micro-batch, the zero-padded ``[micro-batches, numel]``
table is summed over the workers (every row has exactly one non-zero contributor, so the sum is
exact), and every rank adds the rows in global micro-batch order -- the order single-process
training accumulates them -- so the loss trajectory stays bit-identical across
reconfigurations.  ``sync_full_state`` copies model and optimizer state from a source worker to
a lagging or new one.
Parity: ``resihp/runtime/dp_runtime.py:14-85`` (same iteration contract and state sync; the
canonical micro-batch-order reduction is ours).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..comm.comm_manager import GenerationComms, ResilientCommManager
from ..state.rng_data import IndexAddressableSampler
from .optim import Adam


def _flat_grads(params, extra: torch.Tensor) -> torch.Tensor:
    parts = [(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for p in params]
    return torch.cat(parts + [extra.reshape(-1)])


class DataParallelRuntime:
    def __init__(self, cfg, sampler: IndexAddressableSampler, model, comms: GenerationComms,
                 mgr: ResilientCommManager, assignment: list[int], *, hook=None, progress=None,
                 timeout: float = 120.0, canonical: bool = False, num_microbatches: int | None = None,
                 batch_fn=None, loss_fn=None, tokens_fn=None):
        self.cfg, self.sampler, self.model, self.comms, self.mgr = cfg, sampler, model, comms, mgr
        self.assignment = assignment
        self.hook = hook or (lambda it, phase: None)
        self.progress = progress or (lambda **kw: None)
        self.timeout, self.canonical = timeout, canonical
        self.num_microbatches = num_microbatches or sampler.num_microbatches
        if batch_fn is None:  # the MLP reference model
            from .reference_model import global_tokens, microbatch, token_loss

            def batch_fn(it, mb):
                return microbatch(cfg, sampler, it, mb)

            def loss_fn(model_, m):
                return token_loss(model_(m.x), m.y, m.mask)

            def tokens_fn(it):
                return global_tokens(cfg, sampler, it)
        self.batch_fn, self.loss_fn, self.tokens_fn = batch_fn, loss_fn, tokens_fn

    def _all_reduce(self, t: torch.Tensor, what: str) -> None:
        self.mgr.guarded_wait(dist.all_reduce(t, async_op=True), timeout=self.timeout, what=what)

    def run_iteration(self, iteration: int) -> float:
        params = [p for _, p in self.model.named_state().items()]
        dtype = params[0].dtype
        for p in params:
            p.grad = None
        rows: dict[int, torch.Tensor] = {}
        loss_sum = 0.0
        for mb in self.assignment:
            self.hook(iteration, "forward")
            self.progress(iteration=iteration, phase=f"mb{mb}", in_collective=False)
            loss = self.loss_fn(self.model, self.batch_fn(iteration, mb))
            if self.canonical:
                grads = torch.autograd.grad(loss, params, allow_unused=True)
                rows[mb] = torch.cat([(g if g is not None else torch.zeros_like(p)).reshape(-1)
                                      for g, p in zip(grads, params)] + [loss.detach().reshape(1)])
            else:
                loss.backward()
            loss_sum += loss.item()
        self.hook(iteration, "reduce")
        tokens = self.tokens_fn(iteration)
        if self.canonical:
            flat = self._canonical_reduce(rows, params, dtype)
        else:
            flat = _flat_grads(params, torch.tensor([loss_sum], dtype=dtype))
            if self.comms.world_size > 1:
                self.progress(iteration=iteration, phase="grad_allreduce", in_collective=True)
                self._all_reduce(flat, "grad all-reduce")
        sizes = [p.numel() for p in params]
        for p, piece in zip(params, flat[:sum(sizes)].split(sizes)):
            p.grad = (piece.view_as(p) / tokens).clone()
        self.hook(iteration, "step")
        return flat[-1].item() / tokens

    def _canonical_reduce(self, rows: dict[int, torch.Tensor], params, dtype) -> torch.Tensor:
        """Per-micro-batch vectors summed in global micro-batch order (layout-invariant)."""
        width = 1 + sum(p.numel() for p in params)
        table = torch.zeros(self.num_microbatches, width, dtype=dtype)
        for mb, row in rows.items():
            table[mb] = row
        if self.comms.world_size > 1:
            self.progress(in_collective=True, phase="grad_gather")
            self._all_reduce(table, "grad gather")  # x + 0 is exact: every row is reproduced bit for bit
        total = torch.zeros(width, dtype=dtype)
        for row in table:
            total = total + row
        return total


def full_state(opt: Adam, committed_iteration: int) -> tuple[dict[str, torch.Tensor], torch.Tensor]:
    return opt.state_tensors(), torch.tensor([committed_iteration, opt.step_count], dtype=torch.int64)


def sync_full_state(mgr: ResilientCommManager, comms: GenerationComms, my_id: str, sources: dict[str, str], opt: Adam,
                    committed_iteration: int, timeout: float = 120.0) -> int | None:
    """Copy model and optimizer state from each receiver's source to it; returns the adopted
    iteration on receivers and None elsewhere.  Tag 0 carries (iteration, step count), tags 1..
    the state tensors in name order."""
    tensors, header = full_state(opt, committed_iteration)
    names = sorted(tensors)
    works, incoming, in_header = [], None, torch.zeros(2, dtype=torch.int64)
    for dst, src in sorted(sources.items()):
        if my_id == src:
            to = comms.rank_of(dst)
            works.append(dist.isend(header, to, tag=0))
            works += [dist.isend(tensors[n].contiguous(), to, tag=t) for t, n in enumerate(names, start=1)]
        if my_id == dst:
            frm = comms.rank_of(src)
            incoming = {n: torch.empty_like(tensors[n]) for n in names}
            works.append(dist.irecv(in_header, frm, tag=0))
            works += [dist.irecv(incoming[n], frm, tag=t) for t, n in enumerate(names, start=1)]
    for work in works:
        mgr.guarded_wait(work, timeout=timeout, what="state sync")
    if incoming is None:
        return None
    opt.load_state_tensors(incoming, int(in_header[1].item()))
    return int(in_header[0].item())
