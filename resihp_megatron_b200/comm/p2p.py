"""Pipeline-boundary transfers between TP groups of different sizes (interval routing on rows).

* Sequence parallel: sender rank ``i`` owns token rows ``even_split(n, k_src)[i]`` and receiver
  ``j`` needs ``even_split(n, k_dst)[j]``; each overlap goes point to point, no collective.
* Replicated activations (no SP): every sender holds the full tensor, sender ``i`` is only
  responsible for ``even_split(n, k_src)[i]``, so each element crosses the boundary once and the
  receivers reassemble the full tensor with one all-gather inside their TP group.
Works for any pair of TP degrees, including 3 <-> 4.  ``channels`` gives each direction of a rank
pair its own 2-rank group (needed for NCCL FIFO safety).  Pipeline send/recv stays on NCCL
point-to-point by design.  (Reference: ``resihp/comm/hetero_p2p.py:32-112``.)
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..utils.intervals import even_split, overlaps


@dataclass(frozen=True)
class Route:
    src: int
    dst: int
    rows: tuple[int, int]


def boundary_routes(src_ranks: tuple[int, ...], dst_ranks: tuple[int, ...], n_rows: int) -> list[Route]:
    a = even_split(n_rows, len(src_ranks))
    b = even_split(n_rows, len(dst_ranks))
    return [Route(src_ranks[i], dst_ranks[j], iv) for i, j, iv in overlaps(a, b)]


def local_rows(n_rows: int, group_ranks: tuple[int, ...], rank: int) -> tuple[int, int]:
    return even_split(n_rows, len(group_ranks))[group_ranks.index(rank)]


def channel_name(src: int, dst: int) -> str:
    return f"p2p/{src}>{dst}"


def message_tag(base: int, index: int) -> int:
    return (base * 4096 + index) % (2 ** 31 - 1)


class P2PEngine:
    def __init__(self, rank: int, mgr, *, channels: dict[tuple[int, int], object] | None = None,
                 timeout: float = 120.0, device: str = "cpu"):
        self.rank = rank
        self.mgr = mgr
        self.channels = channels
        self.timeout = timeout
        self.device = device

    def _group(self, src: int, dst: int):
        return None if self.channels is None else self.channels[(src, dst)]

    def send(self, local: torch.Tensor, src_ranks: tuple[int, ...], dst_ranks: tuple[int, ...], n_rows: int,
             sequence_parallel: bool, tag: int) -> list:
        """Post the sends of this rank (non-blocking); returns the works to wait on later."""
        works = []
        offset = local_rows(n_rows, src_ranks, self.rank)[0] if sequence_parallel else 0
        for i, rt in enumerate(boundary_routes(src_ranks, dst_ranks, n_rows)):
            if rt.src != self.rank:
                continue
            piece = local.narrow(0, rt.rows[0] - offset, rt.rows[1] - rt.rows[0]).contiguous()
            works.append((dist.isend(piece, rt.dst, group=self._group(rt.src, rt.dst), tag=message_tag(tag, i)),
                          piece))
        return works

    def recv(self, n_rows: int, row_shape: tuple[int, ...], dtype: torch.dtype, src_ranks: tuple[int, ...],
             dst_ranks: tuple[int, ...], sequence_parallel: bool, tag: int, tp_group=None) -> torch.Tensor:
        mine = local_rows(n_rows, dst_ranks, self.rank)
        out = torch.empty((mine[1] - mine[0],) + tuple(row_shape), dtype=dtype, device=self.device)
        pending = []
        for i, rt in enumerate(boundary_routes(src_ranks, dst_ranks, n_rows)):
            if rt.dst != self.rank:
                continue
            buf = torch.empty((rt.rows[1] - rt.rows[0],) + tuple(row_shape), dtype=dtype, device=self.device)
            work = dist.irecv(buf, rt.src, group=self._group(rt.src, rt.dst), tag=message_tag(tag, i))
            pending.append((work, buf, rt.rows))
        for work, buf, rows in pending:
            self.mgr.guarded_wait(work, timeout=self.timeout, what="boundary recv")
            out.narrow(0, rows[0] - mine[0], rows[1] - rows[0]).copy_(buf)
        if sequence_parallel or len(dst_ranks) == 1:
            return out
        return self._gather_rows(out, n_rows, dst_ranks, tp_group)

    def _gather_rows(self, mine: torch.Tensor, n_rows: int, ranks: tuple[int, ...], group) -> torch.Tensor:
        parts = even_split(n_rows, len(ranks))
        width = max(b - a for a, b in parts)
        padded = torch.zeros((width,) + tuple(mine.shape[1:]), dtype=mine.dtype, device=mine.device)
        padded[: mine.shape[0]].copy_(mine)
        bufs = [torch.empty_like(padded) for _ in ranks]
        self.mgr.guarded_wait(dist.all_gather(bufs, padded, group=group, async_op=True), timeout=self.timeout,
                              what="boundary all-gather")
        return torch.cat([buf[: b - a] for buf, (a, b) in zip(bufs, parts)])

    def wait_sends(self, works: list) -> None:
        for work, _ in works:
            self.mgr.guarded_wait(work, timeout=self.timeout, what="boundary send")
