"""Shard-aligned gradient reduction across DP replicas whose TP degrees differ.

For a stage, every replica splits a partitioned dimension of length ``n`` evenly by its own TP
degree; on the common refinement of those splits each interval has exactly one holder per
replica, and those holders all-reduce exactly that slice (one ``dpshard/s{s}/{ranks}`` group
per holder set).  With uniform TP this is the plain DP all-reduce; with TP 4 vs 3 it is the
correct generalisation (pairing ranks by TP index would be wrong).  TP-replicated parameters
are reduced through responsibility slices (rank ``t`` of a TP-``k`` replica reduces
``even_split(numel, k)[t]``) and re-assembled with one all-gather in the TP group; under sequence
parallelism their gradients are partial and are first summed inside the TP group.
(Reference: ``resihp/runtime/hetero_grad_sync.py:34-126``.)
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


class HeteroGradSync:
    def __init__(self, plan: HeteroParallelPlan, comms, mgr, stage: int, replica: int,
                 params: dict[str, torch.Tensor], shards: dict[str, ParamShard], tp_group=None,
                 timeout: float = 120.0):
        self.plan = plan
        self.comms = comms
        self.mgr = mgr
        self.stage = stage
        self.replica = replica
        self.params = params
        self.shards = shards
        self.tp_group = tp_group
        self.timeout = timeout
        g = plan.group(replica, stage)
        me = plan.world[comms.rank]
        self.tp = g.tp
        self.tp_rank = g.slice(g.slice_of(me)).index(me)
        self.peers = plan.tp_slices(stage)
        self._layout = self._build_layout()

    def _build_layout(self) -> dict[str, list[tuple[str, tuple[int, int], tuple[int, int]]]]:
        """group name -> [(key, global interval, local interval)] in a deterministic order."""
        layout: dict[str, list] = {}
        for key in sorted(self.params):
            info = self.shards[key]
            parts = [even_split(info.full_size, len(sl)) for sl in self.peers]
            mine = even_split(info.full_size, self.tp)[self.tp_rank]
            base = mine[0] if info.dim is not None else 0
            for iv in refine(parts):
                if not (mine[0] <= iv[0] and iv[1] <= mine[1]):
                    continue
                holders = tuple(sorted(self.plan.rank(sl[locate(p, iv)]) for sl, p in zip(self.peers, parts)))
                layout.setdefault(dpshard_group_name(self.stage, holders), []).append(
                    (key, iv, (iv[0] - base, iv[1] - base)))
        return dict(sorted(layout.items()))

    def _rows_view(self, key: str) -> torch.Tensor:
        g = self.params[key].grad
        info = self.shards[key]
        return g.reshape(-1) if info.dim is None else g.movedim(info.dim, 0)

    def _wait(self, work, what: str) -> None:
        self.mgr.guarded_wait(work, timeout=self.timeout, what=what)

    def sync(self) -> None:
        for p in self.params.values():
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        if self.tp > 1:
            partial = [k for k in sorted(self.params) if self.shards[k].sp_partial]
            if partial:
                flat = torch.cat([self.params[k].grad.reshape(-1) for k in partial])
                self._wait(dist.all_reduce(flat, group=self.tp_group, async_op=True), "tp partial-grad all-reduce")
                off = 0
                for k in partial:
                    g = self.params[k].grad
                    g.copy_(flat[off:off + g.numel()].view_as(g))
                    off += g.numel()
        for name, entries in self._layout.items():
            pg = self.comms.groups.get(name)
            if pg is None:
                continue
            views = [self._rows_view(k).narrow(0, loc[0], loc[1] - loc[0]) for k, _, loc in entries]
            flat = torch.cat([v.reshape(-1) for v in views])
            self._wait(dist.all_reduce(flat, group=pg, async_op=True), f"grad all-reduce {name}")
            off = 0
            for v in views:
                v.copy_(flat[off:off + v.numel()].view_as(v))
                off += v.numel()
        if self.tp > 1:
            self._regather_replicated()

    def _regather_replicated(self) -> None:
        for k in sorted(self.params):
            if self.shards[k].dim is not None:
                continue
            flat = self.params[k].grad.reshape(-1)
            parts = even_split(flat.numel(), self.tp)
            width = max(b - a for a, b in parts)
            a, b = parts[self.tp_rank]
            mine = torch.zeros(width, dtype=flat.dtype, device=flat.device)
            mine[: b - a].copy_(flat[a:b])
            bufs = [torch.empty_like(mine) for _ in range(self.tp)]
            self._wait(dist.all_gather(bufs, mine, group=self.tp_group, async_op=True), "replicated grad all-gather")
            flat.copy_(torch.cat([buf[: pb - pa] for buf, (pa, pb) in zip(bufs, parts)]))

    def holder_groups(self) -> list[str]:
        return list(self._layout)
