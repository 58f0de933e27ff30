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
    def __init__(self, rank: int, world: int, exchange, device, abort: AbortWord | None = None,
                 barrier_budget_s: float = 60.0):
        self.rank, self.world = rank, world
        self.exchange = exchange
        self.device = torch.device(device)
        self.abort = abort
        self.budget = barrier_budget_s
        self.heap: SymmetricHeap | None = None

    def buffer_factory(self, numel: int):
        """For ``FlatParams(buffer_factory=...)``: zero-filled heap-resident bf16 and grad buffers,
        plus room for this rank's optimizer shard (``opt_factory``), so a later reconfiguration can
        pull master weights and moments from this rank's memory peer to peer."""
        shard = numel // self.world
        self.heap = SymmetricHeap({"grad": (numel, torch.float32), "weight": (numel, torch.bfloat16),
                                   "master": (shard, torch.float32), "exp_avg": (shard, torch.float32),
                                   "exp_avg_sq": (shard, torch.float32)}, self.rank, self.world, self.exchange,
                                  self.device, self.abort)
        return self.heap.tensor("weight"), self.heap.tensor("grad")

    def opt_factory(self, shard_numel: int):
        assert self.heap is not None and self.heap.segments["master"].numel == shard_numel
        return self.heap.tensor("master"), self.heap.tensor("exp_avg"), self.heap.tensor("exp_avg_sq")

    def step(self, P, *, lr, betas, eps, weight_decay, grad_scale: float = 1.0, decoupled: bool = False) -> None:
        """One optimizer step of flat parameters ``P`` (whose buffers came from ``buffer_factory``)."""
        heap = self.heap
        assert heap is not None, "buffers were not allocated by this FusedDataParallel"
        heap.barrier(self.budget)
        ext().dp_step_fused(heap.peer_ptrs("grad"), heap.peer_ptrs("weight"), P.master, P.exp_avg, P.exp_avg_sq,
                            P.shard_lo, float(lr), float(betas[0]), float(betas[1]), float(eps), float(weight_decay),
                            bool(decoupled), int(P.step), float(grad_scale), self.abort.dev if self.abort else 0)
        heap.barrier(self.budget)
        P.grad.zero_()

    def check(self) -> None:
        if self.heap is not None:
            self.heap.check()

    def close(self) -> None:
        if self.heap is not None:
            self.heap.close()
            self.heap = None


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
