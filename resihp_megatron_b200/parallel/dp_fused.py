"""Fused data-parallel gradient reduction + Adam + weight gather on symmetric peer memory.

The flat fp32 gradients and bf16 weights of every rank live in the symmetric heap.  After the
backward of the last micro-batch a bounded barrier makes every rank's gradients visible; one
kernel per rank then, for its own contiguous shard, sums the gradients of all ranks with peer
loads in rank order (deterministic, and identical on every rank), applies Adam to the fp32
master shard, and writes the shard's new bf16 weights into every rank's weight buffer with peer
stores.  A second barrier closes the step (no rank reuses its gradient buffer before every peer
read it, and no rank starts the next forward before all weights landed).  This replaces the
reduce-scatter, the optimizer pass and the all-gather of the NCCL path with one pass over NVLink
(reference call sites C5/C6/C9: ``resihp/runtime/hetero_grad_sync.py:101,121``,
``resihp/runtime/dp_runtime.py:45``).
"""

from __future__ import annotations

import torch

from ..ops._build import ext
from .symm import AbortWord, SymmetricHeap


class FusedDataParallel:
    """Two symmetric heaps per generation: ``state`` (bf16 weights + this rank's fp32 master and
    Adam moments; its signal pad carries the barriers) and ``grads`` (the full fp32 gradient).
    Keeping them apart lets a reconfiguration drop the gradients first and hold only the old and
    new optimizer state at the same time."""

    STATE = ("master", "exp_avg", "exp_avg_sq")

    def __init__(self, rank: int, world: int, exchange, device, abort: AbortWord | None = None,
                 barrier_budget_s: float = 60.0):
        self.rank, self.world = rank, world
        self.exchange = exchange
        self.device = torch.device(device)
        self.abort = abort
        self.budget = barrier_budget_s
        self.state: SymmetricHeap | None = None
        self.grads: SymmetricHeap | None = None

    @property
    def heap(self) -> SymmetricHeap | None:
        """The heap whose signal pad orders the ranks (the state heap)."""
        return self.state

    def alloc_state(self, numel: int) -> None:
        shard = numel // self.world
        self.state = SymmetricHeap({"weight": (numel, torch.bfloat16), "master": (shard, torch.float32),
                                    "exp_avg": (shard, torch.float32), "exp_avg_sq": (shard, torch.float32)},
                                   self.rank, self.world, self.exchange, self.device, self.abort)

    def alloc_grads(self, numel: int) -> None:
        self.grads = SymmetricHeap({"grad": (numel, torch.float32)}, self.rank, self.world, self.exchange,
                                   self.device, self.abort)

    def buffer_factory(self, numel: int):
        """For ``FlatParams(buffer_factory=...)``: zero-filled heap-resident bf16 and grad buffers
        (allocated here unless already allocated)."""
        if self.state is None:
            self.alloc_state(numel)
        if self.grads is None:
            self.alloc_grads(numel)
        return self.state.tensor("weight"), self.grads.tensor("grad")

    def opt_factory(self, shard_numel: int):
        assert self.state is not None and self.state.segments["master"].numel == shard_numel
        return tuple(self.state.tensor(k) for k in self.STATE)

    def step(self, P, *, lr, betas, eps, weight_decay, grad_scale: float = 1.0, decoupled: bool = False) -> None:
        """One optimizer step of flat parameters ``P`` (whose buffers came from ``buffer_factory``)."""
        assert self.state is not None and self.grads is not None, "buffers were not allocated here"
        self.state.barrier(self.budget)
        ext().dp_step_fused(self.grads.peer_ptrs("grad"), self.state.peer_ptrs("weight"), P.master, P.exp_avg,
                            P.exp_avg_sq, P.shard_lo, float(lr), float(betas[0]), float(betas[1]), float(eps),
                            float(weight_decay), bool(decoupled), int(P.step), float(grad_scale),
                            self.abort.dev if self.abort else 0)
        self.state.barrier(self.budget)
        P.grad.zero_()

    def check(self) -> None:
        if self.state is not None:
            self.state.check()

    def close_grads(self) -> None:
        if self.grads is not None:
            self.grads.close()
            self.grads = None

    def close(self) -> None:
        self.close_grads()
        if self.state is not None:
            self.state.close()
            self.state = None


def reshard_pull_plan(old_world: int, old_shard: int, old_ptrs: dict[str, list[int]], new_lo: int, new_hi: int,
                      new_ptrs: dict[str, int], old_numel: int) -> list[int]:
    """Flat (src, dst, bytes) triples that fill this rank's new optimizer shard ``[new_lo, new_hi)``
    from the old owners' shards (old owner ``o`` held ``[o * old_shard, (o + 1) * old_shard)``).
    Elements past the old flat size are padding and stay zero."""
    triples: list[int] = []
    for o in range(old_world):
        a = max(new_lo, o * old_shard)
        b = min(new_hi, (o + 1) * old_shard, old_numel)
        if a >= b:
            continue
        for seg in ("master", "exp_avg", "exp_avg_sq"):
            triples += [old_ptrs[seg][o] + (a - o * old_shard) * 4, new_ptrs[seg] + (a - new_lo) * 4, (b - a) * 4]
    return triples
