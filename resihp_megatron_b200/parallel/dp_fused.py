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
    """Symmetric heap per job: the full fp32 gradient, the full bf16 weights and the fp32 optimizer
    shard (master weights + both Adam moments) of this rank.

    With ``spare_bank`` (default when there are at least 4 ranks) the optimizer state has two
    banks, each sized for a world one rank smaller, and the gradient / weight segments are sized
    for any shard count up to the world size.  A live shrink then moves only the optimizer shards
    -- peer to peer, from the old owners' current bank into each survivor's other bank -- and keeps
    every buffer and every mapping: the weights and gradients do not depend on the shard layout.
    Without a spare bank a shrink builds the next generation's heap instead."""

    STATE = ("master", "exp_avg", "exp_avg_sq")

    def __init__(self, rank: int, world: int, exchange, device, abort: AbortWord | None = None,
                 barrier_budget_s: float = 60.0, numel_cap: int | None = None, spare_bank: bool | None = None):
        self.rank, self.world = rank, world
        self.exchange = exchange
        self.device = torch.device(device)
        self.abort = abort
        self.budget = barrier_budget_s
        self.numel_cap = numel_cap
        self.banks = 2 if (spare_bank if spare_bank is not None else world >= 4) else 1
        self.bank = 0
        self.heap: SymmetricHeap | None = None
        self.numel = 0
        self.ring = None  # DeviceRing: one timing record per fused step

    def _shard_cap(self) -> int:
        from ..models.params import ALIGN

        ranks = self.world - 1 if self.banks == 2 else self.world
        cap = self.numel_cap or self.numel
        return -(-cap // (ranks * ALIGN)) * ALIGN

    def buffer_factory(self, numel: int):
        """For ``FlatParams(buffer_factory=...)``: zero-filled heap-resident bf16 and grad views."""
        if self.heap is None:
            self.numel = numel
            cap = max(self.numel_cap or numel, numel)
            self.numel_cap = cap
            segs: dict = {"grad": (cap, torch.float32), "weight": (cap, torch.bfloat16)}
            for b in range(self.banks):
                for k in self.STATE:
                    segs[f"{k}{b}"] = (self._shard_cap(), torch.float32)
            self.heap = SymmetricHeap(segs, self.rank, self.world, self.exchange, self.device, self.abort)
        assert numel <= self.numel_cap
        self.numel = numel
        return self.heap.tensor("weight")[:numel], self.heap.tensor("grad")[:numel]

    def opt_factory(self, shard_numel: int):
        assert self.heap is not None and shard_numel <= self.heap.segments[f"master{self.bank}"].numel
        return tuple(self.heap.tensor(f"{k}{self.bank}")[:shard_numel] for k in self.STATE)

    def state_ptrs(self, bank: int) -> dict[str, list[int]]:
        return {k: self.heap.peer_ptrs(f"{k}{bank}") for k in self.STATE}

    def step(self, P, *, lr, betas, eps, weight_decay, grad_scale: float = 1.0, decoupled: bool = False) -> None:
        """One optimizer step of flat parameters ``P`` (whose buffers came from ``buffer_factory``)."""
        heap = self.heap
        assert heap is not None, "buffers were not allocated here"
        heap.barrier(self.budget)
        ext().dp_step_fused(heap.peer_ptrs("grad"), heap.peer_ptrs("weight"), P.master, P.exp_avg, P.exp_avg_sq,
                            P.shard_lo, float(lr), float(betas[0]), float(betas[1]), float(eps), float(weight_decay),
                            bool(decoupled), int(P.step), float(grad_scale), self.abort.dev if self.abort else 0,
                            self.ring.dev if self.ring else 0, self.ring.capacity if self.ring else 0,
                            self.ring.stamp.data_ptr() if self.ring else 0)
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
