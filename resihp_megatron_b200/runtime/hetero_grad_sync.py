"""Shard-aligned gradient reduction across DP replicas whose TP degrees differ.

For one stage, every replica splits a partitioned dimension of length ``n`` evenly by its own
TP degree.  On the common refinement of those splits each interval has exactly one holder per
replica, and exactly those holders all-reduce that interval (one ``dpshard/s{s}/{ranks}`` group
per holder set).  With uniform TP this is the plain DP all-reduce; with, say, TP4 next to TP3 it
is the correct generalisation (pairing ranks by TP index would not be).  A TP-replicated
parameter is reduced through responsibility slices -- TP rank ``t`` of a TP-``k`` replica
reduces ``even_split(numel, k)[t]`` -- and re-assembled with one all-gather in the TP group;
under sequence parallelism its gradient is a partial sum over token shards and is first summed
inside the TP group.
Parity: ``resihp/runtime/hetero_grad_sync.py:34-126`` (same holder sets and reduction steps).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..plan.hetero_plan import HeteroParallelPlan, dpshard_group_name
from ..utils.intervals import even_split, locate, refine


@dataclass(frozen=True)
class ParamShard:
    key: str
    dim: int | None
    full_size: int
    sp_partial: bool = False


def _packed_all_reduce(views: list[torch.Tensor], issue, what: str) -> None:
    """All-reduce several tensor views as one flat buffer and write the sums back."""
    flat = torch.cat([v.reshape(-1) for v in views])
    issue(flat, what)
    offset = 0
    for v in views:
        v.copy_(flat[offset:offset + v.numel()].view_as(v))
        offset += v.numel()


class HeteroGradSync:
    def __init__(self, plan: HeteroParallelPlan, comms, mgr, stage: int, replica: int,
                 params: dict[str, torch.Tensor], shards: dict[str, ParamShard], tp_group=None,
                 timeout: float = 120.0):
        self.plan, self.comms, self.mgr = plan, comms, mgr
        self.stage, self.replica = stage, replica
        self.params, self.shards = params, shards
        self.tp_group, self.timeout = tp_group, timeout
        group = plan.group(replica, stage)
        me = plan.world[comms.rank]
        self.tp = group.tp
        self.tp_rank = group.slice(group.slice_of(me)).index(me)
        self.peers = plan.tp_slices(stage)
        self._buckets = self._plan_buckets()

    def _plan_buckets(self) -> dict[str, list[tuple[str, tuple[int, int], tuple[int, int]]]]:
        """Reduction group name -> ``(key, global interval, local interval)`` of the pieces this rank
        reduces in it, groups in name order (the same order on every member)."""
        buckets: dict[str, list] = {}
        for key in sorted(self.params):
            info = self.shards[key]
            splits = [even_split(info.full_size, len(peer)) for peer in self.peers]
            lo, hi = even_split(info.full_size, self.tp)[self.tp_rank]
            offset = lo if info.dim is not None else 0
            for piece in refine(splits):
                if piece[0] < lo or piece[1] > hi:
                    continue  # another TP rank of this replica reduces it
                holders = sorted(self.plan.rank(peer[locate(split, piece)]) for peer, split in zip(self.peers, splits))
                name = dpshard_group_name(self.stage, tuple(holders))
                buckets.setdefault(name, []).append((key, piece, (piece[0] - offset, piece[1] - offset)))
        return {name: buckets[name] for name in sorted(buckets)}

    def holder_groups(self) -> list[str]:
        return list(self._buckets)

    def _issue(self, group):
        def run(flat: torch.Tensor, what: str) -> None:
            self.mgr.guarded_wait(dist.all_reduce(flat, group=group, async_op=True), timeout=self.timeout, what=what)

        return run

    def _rows(self, key: str) -> torch.Tensor:
        """The gradient with its partitioned dimension first (flattened when replicated)."""
        grad, dim = self.params[key].grad, self.shards[key].dim
        return grad.reshape(-1) if dim is None else grad.movedim(dim, 0)

    def sync(self) -> None:
        for p in self.params.values():
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        partial = [self.params[k].grad for k in sorted(self.params) if self.shards[k].sp_partial]
        if self.tp > 1 and partial:
            _packed_all_reduce(partial, self._issue(self.tp_group), "tp partial-grad all-reduce")
        for name, pieces in self._buckets.items():
            group = self.comms.groups.get(name)
            if group is None:
                continue  # a holder set of one: nothing to reduce
            views = [self._rows(key).narrow(0, a, b - a) for key, _, (a, b) in pieces]
            _packed_all_reduce(views, self._issue(group), f"grad all-reduce {name}")
        if self.tp > 1:
            for key in (k for k in sorted(self.params) if self.shards[k].dim is None):
                self._reassemble(self.params[key].grad.reshape(-1))

    def _reassemble(self, flat: torch.Tensor) -> None:
        """Every TP rank reduced its responsibility slice of a replicated gradient: gather them."""
        slices = even_split(flat.numel(), self.tp)
        width = max(b - a for a, b in slices)
        lo, hi = slices[self.tp_rank]
        padded = torch.zeros(width, dtype=flat.dtype, device=flat.device)
        padded[:hi - lo] = flat[lo:hi]
        gathered = [torch.empty_like(padded) for _ in slices]
        self.mgr.guarded_wait(dist.all_gather(gathered, padded, group=self.tp_group, async_op=True),
                              timeout=self.timeout, what="replicated grad all-gather")
        for part, (a, b) in zip(gathered, slices):
            flat[a:b] = part[:b - a]
