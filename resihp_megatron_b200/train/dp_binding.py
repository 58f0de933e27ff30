"""Binds the replica-level DP runtime to the resilient loop (any float model + Adam).

Recovery, in order: a rank holding the target iteration's reduced gradients steps locally
(roll-forward); every rank that needs state receives the model and Adam state from the source
the planner assigned it (same node first); with ``restore == "checkpoint"`` the newest complete
T2 checkpoint is loaded instead.  T1 host snapshots are taken every ``snapshot_interval``
iterations and mirrored to the ring buddy; rank 0 writes T2 checkpoints.  ``canonical=True``
selects the layout-invariant gradient reduction in micro-batch order, which keeps the loss
bit-identical across reconfigurations.
Parity: ``resihp/train/dp_binding.py:16-105`` (same recovery order, snapshot and checkpoint use).
"""

from __future__ import annotations

import torch

from ..comm.comm_manager import GenerationComms, ResilientCommManager
from ..comm.group_spec import GroupSpec
from ..control.worker_client import WorkerClient
from ..runtime.dp_runtime import DataParallelRuntime, sync_full_state
from ..runtime.optim import Adam
from ..state.checkpoint import SliceCheckpointer, SliceMeta
from ..state.redundancy import HostSnapshotManager, exchange_snapshot_with_buddy
from ..state.transaction import TransactionManager

_WHOLE = (0, 1)  # a replicated tensor is checkpointed as one slice


class DPBinding:
    def __init__(self, cfg, sampler, model, opt: Adam, mgr: ResilientCommManager, client: WorkerClient, *,
                 injector=None, snapshots: HostSnapshotManager | None = None, replicate_snapshots: bool = True,
                 checkpointer: SliceCheckpointer | None = None, checkpoint_interval: int = 0, timeout: float = 120.0,
                 canonical: bool = False, runtime_kwargs: dict | None = None):
        self.cfg, self.sampler, self.model, self.opt = cfg, sampler, model, opt
        self.mgr, self.client, self.injector = mgr, client, injector
        self.snapshots, self.replicate_snapshots = snapshots, replicate_snapshots
        self.checkpointer, self.checkpoint_interval = checkpointer, checkpoint_interval
        self.timeout, self.canonical = timeout, canonical
        self.runtime_kwargs = dict(runtime_kwargs or {})
        self.me = client.worker_id

    def group_specs(self, world: list[str], payload: dict) -> list[GroupSpec]:
        return []  # everything runs on the world group

    def build_runtime(self, comms: GenerationComms, payload: dict) -> DataParallelRuntime:
        return DataParallelRuntime(self.cfg, self.sampler, self.model, comms, self.mgr, payload["assignment"][self.me],
                                   hook=None if self.injector is None else self.injector.on_hook,
                                   progress=self.client.set_progress, timeout=self.timeout, canonical=self.canonical,
                                   num_microbatches=payload.get("num_microbatches"), **self.runtime_kwargs)

    def recover(self, comms: GenerationComms, payload: dict, txm: TransactionManager) -> None:
        recovery = payload["recovery"]
        if recovery.get("restore") == "checkpoint":
            restored = self._load_checkpoint()
            if restored is None:
                raise RuntimeError("checkpoint restore requested but no complete checkpoint exists")
            txm.adopt(restored)
        else:
            if txm.has_reduced_grads and self.me in recovery["local_step"]:
                self.opt.step()
                txm.adopt(recovery["target_iteration"])
            received = sync_full_state(self.mgr, comms, self.me, recovery["sources"], self.opt,
                                       txm.committed_iteration, timeout=self.timeout)
            if received is not None:
                txm.adopt(received)
        txm.discard()
        self.opt.zero_grad()

    def optimizer_step(self) -> None:
        if self.snapshots is not None:
            self.snapshots.fence()  # a snapshot copy in flight must finish before the update
        self.opt.step()

    def discard_grads(self) -> None:
        self.opt.zero_grad()

    def after_commit(self, iteration: int, comms: GenerationComms) -> None:
        if self.snapshots is not None and self.snapshots.due(iteration):
            self._snapshot(iteration, comms)
        every = self.checkpoint_interval
        if self.checkpointer is not None and every and (iteration + 1) % every == 0 and comms.rank == 0:
            pieces = [(SliceMeta(name, tuple(t.shape), None, _WHOLE), {"value": t})
                      for name, t in self.opt.state_tensors().items()]
            self.checkpointer.save(iteration, self.me, pieces, extra={"step_count": self.opt.step_count},
                                   blocking=True)

    def _snapshot(self, iteration: int, comms: GenerationComms) -> None:
        tensors = self.opt.state_tensors()
        self.snapshots.snapshot(iteration, tensors, blocking=True)
        if not self.replicate_snapshots or comms.world_size < 2:
            return
        ring, me = list(comms.world), comms.rank
        successor, predecessor = ring[(me + 1) % len(ring)], ring[me - 1]
        held_it, held = exchange_snapshot_with_buddy(self.mgr, comms, self.snapshots.latest(), send_to=successor,
                                                     recv_from=predecessor, template=tensors, timeout=self.timeout)
        self.snapshots.hold_for(predecessor, held_it, held)

    def _load_checkpoint(self) -> int | None:
        if self.checkpointer is None:
            return None
        shapes = {name: (tuple(t.shape), None) for name, t in self.opt.state_tensors().items()}
        iteration = self.checkpointer.latest_complete(shapes)
        if iteration is None:
            return None
        wanted = [SliceMeta(name, shape, None, _WHOLE) for name, (shape, _) in shapes.items()]
        values = self.checkpointer.load(iteration, wanted, kinds=("value",))
        any_owner = next(self.checkpointer._dir(iteration).glob("*.pt"))
        step_count = torch.load(any_owner, weights_only=False)["extra"]["step_count"]
        self.opt.load_state_tensors({name: v["value"] for name, v in values.items()}, step_count)
        return iteration

    def try_resume(self, txm: TransactionManager) -> None:
        restored = self._load_checkpoint()
        if restored is not None:
            txm.adopt(restored)
