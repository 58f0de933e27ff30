"""Redundancy tiers of training state.

* **T0, live replicas.**  Parameters live on every DP replica of a stage.  With a sharded
  optimizer and the DP group split into several optimizer instances, every optimizer shard has
  a twin holder in each instance (``distopt_twin_holders``).  No rollback.
* **T1, host snapshots** every ``interval`` iterations: pinned host buffers filled on a side
  stream (``fence()`` orders the next in-place update after the copy), mirrored to a buddy on the
  next node of a ring.  Rolls back at most ``interval`` iterations; survives the loss of every
  live copy of a shard.
* **T2, sliced checkpoints** that reshard on load (``checkpoint.py``).
Parity: ``resihp/state/redundancy.py:21-163`` (same tiers, snapshot protocol and ring exchange).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Callable

import torch


def distopt_twin_holders(dp_members: list[str], num_instances: int) -> dict[str, list[str]]:
    """Holders of every optimizer shard when the DP group is cut into ``num_instances``
    consecutive instances: shard ``j`` sits at position ``j`` of each instance."""
    if num_instances < 1 or len(dp_members) % num_instances:
        raise ValueError(f"DP size {len(dp_members)} is not divisible by {num_instances} instances")
    per = len(dp_members) // num_instances
    instances = [dp_members[k:k + per] for k in range(0, len(dp_members), per)]
    return {f"shard{j}": [inst[j] for inst in instances] for j in range(per)}


@dataclass
class HolderMap:
    holders: dict[str, list[str]]

    def lost(self, failed: set[str]) -> list[str]:
        """Shards none of whose holders survived."""
        return sorted(shard for shard, hs in self.holders.items() if set(hs) <= failed)

    def survivors(self, key: str, failed: set[str]) -> list[str]:
        return [h for h in self.holders[key] if h not in failed]

    def node_diverse(self, node_of: Callable[[str], str]) -> bool:
        """Every shard with several holders has them on at least two nodes."""
        return all(len(set(map(node_of, hs))) > 1 for hs in self.holders.values() if len(hs) > 1)


class HostSnapshotManager:
    """Asynchronous host-memory snapshots of a flat ``name -> tensor`` state dict."""

    def __init__(self, interval: int, keep: int = 1):
        self.interval, self.keep = interval, keep
        self._history: list[tuple[int, dict[str, torch.Tensor]]] = []  # oldest first, at most ``keep``
        self._buddies: dict[str, tuple[int, dict[str, torch.Tensor]]] = {}
        self._mu = threading.Lock()
        self._publisher: threading.Thread | None = None
        self._copied: torch.cuda.Event | None = None

    def due(self, iteration: int) -> bool:
        return self.interval > 0 and (iteration + 1) % self.interval == 0

    def _publish(self, iteration: int, staged: dict[str, torch.Tensor], side) -> None:
        if side is not None:
            side.synchronize()
        with self._mu:
            self._history = (self._history + [(iteration, staged)])[-self.keep:]

    def snapshot(self, iteration: int, state: dict[str, torch.Tensor], blocking: bool = False) -> None:
        """CPU tensors are cloned at once; CUDA tensors are copied into pinned host memory on a
        side stream -- call ``fence()`` before the next in-place update of ``state``."""
        self.wait()
        on_gpu = any(t.is_cuda for t in state.values())
        side = torch.cuda.Stream() if on_gpu else None
        if side is not None:
            side.wait_stream(torch.cuda.current_stream())
        staged = {}
        for name, t in state.items():
            if not t.is_cuda:
                staged[name] = t.detach().clone()
                continue
            with torch.cuda.stream(side):
                host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                host.copy_(t.detach(), non_blocking=True)
            staged[name] = host
        if side is not None:
            self._copied = torch.cuda.Event()
            self._copied.record(side)
        if blocking or side is None:
            self._publish(iteration, staged, side)
            return
        self._publisher = threading.Thread(target=self._publish, args=(iteration, staged, side), name="snapshot",
                                           daemon=True)
        self._publisher.start()

    def fence(self) -> None:
        """Make the current stream wait for the last snapshot's device-to-host copies."""
        event, self._copied = self._copied, None
        if event is not None:
            torch.cuda.current_stream().wait_event(event)

    def maybe_snapshot(self, iteration: int, state_fn: Callable[[], dict[str, torch.Tensor]]) -> bool:
        if self.due(iteration):
            self.snapshot(iteration, state_fn(), blocking=True)
            return True
        return False

    def wait(self) -> None:
        worker, self._publisher = self._publisher, None
        if worker is not None:
            worker.join()

    def latest(self) -> tuple[int, dict[str, torch.Tensor]] | None:
        self.wait()
        with self._mu:
            return self._history[-1] if self._history else None

    def at(self, iteration: int) -> dict[str, torch.Tensor] | None:
        self.wait()
        with self._mu:
            return next((snap for it, snap in self._history if it == iteration), None)

    def hold_for(self, owner: str, iteration: int, state: dict[str, torch.Tensor]) -> None:
        """Keep a buddy's snapshot (received over the replication ring)."""
        with self._mu:
            self._buddies[owner] = (iteration, state)

    def held(self, owner: str) -> tuple[int, dict[str, torch.Tensor]] | None:
        with self._mu:
            return self._buddies.get(owner)


def exchange_snapshot_with_buddy(mgr, comms, mine: tuple[int, dict[str, torch.Tensor]], send_to: str,
                                 recv_from: str, template: dict[str, torch.Tensor], group=None,
                                 timeout: float = 60.0) -> tuple[int, dict[str, torch.Tensor]]:
    """Ring replication: send my newest snapshot to ``send_to`` and receive ``recv_from``'s
    (its tensors shaped like ``template``); tag 0 carries the iteration, tags 1.. the tensors in
    name order."""
    import torch.distributed as dist

    iteration, state = mine
    to, frm = comms.rank_of(send_to), comms.rank_of(recv_from)
    out_hdr, in_hdr = torch.tensor([iteration], dtype=torch.int64), torch.zeros(1, dtype=torch.int64)
    received = {name: torch.empty_like(t, device="cpu") for name, t in sorted(template.items())}
    works = [dist.isend(out_hdr, to, group=group, tag=0), dist.irecv(in_hdr, frm, group=group, tag=0)]
    works += [dist.isend(state[name].contiguous(), to, group=group, tag=tag)
              for tag, name in enumerate(sorted(state), start=1)]
    works += [dist.irecv(received[name], frm, group=group, tag=tag) for tag, name in enumerate(received, start=1)]
    for work in works:
        mgr.guarded_wait(work, timeout=timeout, what="snapshot replication")
    return int(in_hdr.item()), received
