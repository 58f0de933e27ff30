"""State redundancy tiers.

* T0 -- live replicas: parameters live on every DP replica of a stage; with a sharded optimizer
  the optimizer shard has twin holders when the DP group is split into several optimizer
  instances (``distopt_twin_holders``).  Zero rollback.
* T1 -- host-memory snapshots every ``interval`` iterations (pinned host buffers filled on a
  side stream; ``fence()`` orders the next in-place update after the copy), replicated to a
  buddy on another node over a ring.  Rollback <= interval iterations; covers the loss of every
  live copy of a shard.
* T2 -- persistent sliced checkpoints that reshard on load (``checkpoint.py``).
(Reference: ``resihp/state/redundancy.py:21-163``.)
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Callable

import torch


def distopt_twin_holders(dp_members: list[str], num_instances: int) -> dict[str, list[str]]:
    """Holders of each optimizer shard when the DP group is cut into ``num_instances``
    contiguous instances: shard ``j`` lives at position ``j`` of every instance."""
    d = len(dp_members)
    if num_instances < 1 or d % num_instances:
        raise ValueError(f"DP size {d} is not divisible by {num_instances} instances")
    per = d // num_instances
    return {f"shard{j}": [dp_members[i * per + j] for i in range(num_instances)] for j in range(per)}


@dataclass
class HolderMap:
    holders: dict[str, list[str]]

    def lost(self, failed: set[str]) -> list[str]:
        return sorted(k for k, hs in self.holders.items() if all(h in failed for h in hs))

    def survivors(self, key: str, failed: set[str]) -> list[str]:
        return [h for h in self.holders[key] if h not in failed]

    def node_diverse(self, node_of: Callable[[str], str]) -> bool:
        return all(len({node_of(h) for h in hs}) > 1 for hs in self.holders.values() if len(hs) > 1)


class HostSnapshotManager:
    """Asynchronous host-memory snapshots of a flat ``name -> tensor`` state dict."""

    def __init__(self, interval: int, keep: int = 1):
        self.interval = interval
        self.keep = keep
        self._snaps: list[tuple[int, dict[str, torch.Tensor]]] = []
        self._held: dict[str, tuple[int, dict[str, torch.Tensor]]] = {}
        self._thread: threading.Thread | None = None
        self._lock = threading.Lock()
        self._copy_done = None
        self._pinned: dict[str, torch.Tensor] = {}

    def due(self, iteration: int) -> bool:
        return self.interval > 0 and (iteration + 1) % self.interval == 0

    def _host_buffer(self, k: str, v: torch.Tensor) -> torch.Tensor:
        buf = self._pinned.get(k)
        if buf is None or buf.shape != v.shape or buf.dtype != v.dtype:
            buf = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
        return buf

    def snapshot(self, iteration: int, state: dict[str, torch.Tensor], blocking: bool = False) -> None:
        """CPU tensors are cloned now; CUDA tensors are copied to pinned host memory on a side
        stream -- call ``fence()`` before the next in-place update of ``state``."""
        self.wait()
        side = None
        if any(v.is_cuda for v in state.values()):
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
        staged: dict[str, torch.Tensor] = {}
        for k, v in state.items():
            if v.is_cuda:
                with torch.cuda.stream(side):
                    buf = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
                    buf.copy_(v.detach(), non_blocking=True)
                staged[k] = buf
            else:
                staged[k] = v.detach().clone()
        if side is not None:
            self._copy_done = torch.cuda.Event()
            self._copy_done.record(side)

        def publish() -> None:
            if side is not None:
                side.synchronize()
            with self._lock:
                self._snaps.append((iteration, staged))
                self._snaps = self._snaps[-self.keep:]

        if blocking or side is None:
            publish()
        else:
            self._thread = threading.Thread(target=publish, name="snapshot", daemon=True)
            self._thread.start()

    def fence(self) -> None:
        if self._copy_done is not None:
            torch.cuda.current_stream().wait_event(self._copy_done)
            self._copy_done = None

    def maybe_snapshot(self, iteration: int, state_fn: Callable[[], dict[str, torch.Tensor]]) -> bool:
        if not self.due(iteration):
            return False
        self.snapshot(iteration, state_fn(), blocking=True)
        return True

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None

    def latest(self) -> tuple[int, dict[str, torch.Tensor]] | None:
        self.wait()
        with self._lock:
            return self._snaps[-1] if self._snaps else None

    def at(self, iteration: int) -> dict[str, torch.Tensor] | None:
        self.wait()
        with self._lock:
            for it, s in self._snaps:
                if it == iteration:
                    return s
        return None

    def hold_for(self, owner: str, iteration: int, state: dict[str, torch.Tensor]) -> None:
        """Keep a buddy's snapshot (received over the replication ring)."""
        with self._lock:
            self._held[owner] = (iteration, state)

    def held(self, owner: str) -> tuple[int, dict[str, torch.Tensor]] | None:
        with self._lock:
            return self._held.get(owner)


def exchange_snapshot_with_buddy(mgr, comms, mine: tuple[int, dict[str, torch.Tensor]], send_to: str,
                                 recv_from: str, template: dict[str, torch.Tensor], group=None,
                                 timeout: float = 60.0) -> tuple[int, dict[str, torch.Tensor]]:
    """Ring replication: send my snapshot to ``send_to``, receive ``recv_from``'s (shapes from
    ``template``)."""
    import torch.distributed as dist

    it, state = mine
    dst, src = comms.rank_of(send_to), comms.rank_of(recv_from)
    hdr = torch.tensor([it], dtype=torch.int64)
    rhdr = torch.zeros(1, dtype=torch.int64)
    works = [dist.isend(hdr, dst, group=group, tag=0), dist.irecv(rhdr, src, group=group, tag=0)]
    got = {k: torch.empty_like(v, device="cpu") for k, v in sorted(template.items())}
    for i, k in enumerate(sorted(state)):
        works.append(dist.isend(state[k].contiguous(), dst, group=group, tag=i + 1))
    for i, k in enumerate(sorted(got)):
        works.append(dist.irecv(got[k], src, group=group, tag=i + 1))
    for w in works:
        mgr.guarded_wait(w, timeout=timeout, what="snapshot replication")
    return int(rhdr.item()), got
