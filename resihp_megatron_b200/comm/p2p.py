"""Pipeline-boundary transfers between TP groups of different sizes: interval routing on rows.

* **Sequence parallel:** sender rank ``i`` owns token rows ``even_split(n, k_src)[i]`` and
  receiver ``j`` needs ``even_split(n, k_dst)[j]``; every overlap goes point to point, with no
  collective.
* **Replicated activations (no SP):** every sender holds the whole tensor but sends only its
  share ``even_split(n, k_src)[i]``, so each element crosses the boundary once, and the
  receivers reassemble the whole tensor with one all-gather inside their TP group.

Any pair of TP degrees works, 3 <-> 4 included.  ``channels`` gives every direction of a rank
pair its own 2-rank group, which NCCL needs for FIFO safety.  Pipeline send / recv stays on NCCL
point-to-point by design.
Parity: ``resihp/comm/hetero_p2p.py:32-112`` (same routing rules and channel names).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..utils.intervals import even_split, overlaps

_TAG_LIMIT = 2 ** 31 - 1


@dataclass(frozen=True)
class Route:
    src: int
    dst: int
    rows: tuple[int, int]


def boundary_routes(src_ranks: tuple[int, ...], dst_ranks: tuple[int, ...], n_rows: int) -> list[Route]:
    """One route per overlap of a sender's rows with a receiver's rows, in a fixed order."""
    sent = even_split(n_rows, len(src_ranks))
    wanted = even_split(n_rows, len(dst_ranks))
    return [Route(src_ranks[i], dst_ranks[j], rows) for i, j, rows in overlaps(sent, wanted)]


def local_rows(n_rows: int, group_ranks: tuple[int, ...], rank: int) -> tuple[int, int]:
    return even_split(n_rows, len(group_ranks))[group_ranks.index(rank)]


def channel_name(src: int, dst: int) -> str:
    return f"p2p/{src}>{dst}"


def message_tag(base: int, index: int) -> int:
    """Tag of route ``index`` of a message whose base tag is ``base``."""
    return ((base << 12) + index) % _TAG_LIMIT


class P2PEngine:
    def __init__(self, rank: int, mgr, *, channels: dict[tuple[int, int], object] | None = None,
                 timeout: float = 120.0, device: str = "cpu"):
        self.rank, self.mgr, self.channels = rank, mgr, channels
        self.timeout, self.device = timeout, device

    def _channel(self, route: Route):
        return self.channels[(route.src, route.dst)] if self.channels is not None else None

    def _await(self, work, what: str) -> None:
        self.mgr.guarded_wait(work, timeout=self.timeout, what=what)

    def send(self, local: torch.Tensor, src_ranks: tuple[int, ...], dst_ranks: tuple[int, ...], n_rows: int,
             sequence_parallel: bool, tag: int) -> list:
        """Post this rank's sends without blocking; returns ``(work, buffer)`` pairs to wait on."""
        first_row = local_rows(n_rows, src_ranks, self.rank)[0] if sequence_parallel else 0
        posted = []
        for i, route in enumerate(boundary_routes(src_ranks, dst_ranks, n_rows)):
            if route.src != self.rank:
                continue
            lo, hi = route.rows
            piece = local[lo - first_row:hi - first_row].contiguous()
            posted.append((dist.isend(piece, route.dst, group=self._channel(route), tag=message_tag(tag, i)), piece))
        return posted

    def recv(self, n_rows: int, row_shape: tuple[int, ...], dtype: torch.dtype, src_ranks: tuple[int, ...],
             dst_ranks: tuple[int, ...], sequence_parallel: bool, tag: int, tp_group=None) -> torch.Tensor:
        lo, hi = local_rows(n_rows, dst_ranks, self.rank)
        mine = torch.empty((hi - lo, *row_shape), dtype=dtype, device=self.device)
        arriving = []
        for i, route in enumerate(boundary_routes(src_ranks, dst_ranks, n_rows)):
            if route.dst == self.rank:
                a, b = route.rows
                arriving.append((dist.irecv(mine[a - lo:b - lo], route.src, group=self._channel(route),
                                            tag=message_tag(tag, i)), route))
        for work, _ in arriving:
            self._await(work, "boundary recv")
        if sequence_parallel or len(dst_ranks) == 1:
            return mine
        return self._assemble(mine, n_rows, dst_ranks, tp_group)

    def _assemble(self, mine: torch.Tensor, n_rows: int, ranks: tuple[int, ...], group) -> torch.Tensor:
        """All-gather every TP rank's share (padded to the widest) and trim back to ``n_rows``."""
        shares = even_split(n_rows, len(ranks))
        width = max(b - a for a, b in shares)
        padded = mine.new_zeros((width, *mine.shape[1:]))
        padded[:mine.shape[0]] = mine
        gathered = [torch.empty_like(padded) for _ in ranks]
        self._await(dist.all_gather(gathered, padded, group=group, async_op=True), "boundary all-gather")
        return torch.cat([g[:b - a] for g, (a, b) in zip(gathered, shares)])

    def wait_sends(self, works: list) -> None:
        for work, _buffer in works:
            self._await(work, "boundary send")
