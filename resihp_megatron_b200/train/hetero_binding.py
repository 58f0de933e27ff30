"""Binds the dynamic hybrid-parallel runtime (float64 reference model) to the resilient loop.

Between generations the committed plan's state is moved into the new plan's layout -- TP
resharding, layers changing stage, lost replicas, fp8 amax histories -- by the slice-level
transfer engine, reading only from ranks that are up to date or can roll forward locally.  The
committed generation's state stays untouched until the new one commits, so a reconfiguration
interrupted by another failure restarts from intact state.  T2 checkpoints store every rank's
logical slices and restore into any later layout.
Parity: ``resihp/train/hetero_binding.py:48-192`` (same recovery paths and checkpoint use).
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from ..comm.comm_manager import GenerationComms, ResilientCommManager
from ..comm.group_spec import GroupSpec
from ..control.worker_client import WorkerClient
from ..plan.hetero_plan import HeteroParallelPlan
from ..plan.ir import Schedule, schedule_from_json
from ..runtime.hetero_runtime import HeteroRuntime, build_stage_module, channel_specs, reference_partition_sizes
from ..runtime.optim import Adam
from ..runtime.reference_model import RefModelConfig
from ..state.checkpoint import SliceCheckpointer, SliceMeta
from ..state.layer_registry import device_layout, holdings, reference_layer_of, reference_specs
from ..state.rng_data import IndexAddressableSampler
from ..state.transaction import TransactionManager
from ..state.transfer_engine import LocalState, execute_transfers
from ..state.transfer_plan import plan_transfers

KINDS = ("param", "exp_avg", "exp_avg_sq")


@dataclass
class _Generation:
    """The model, optimizer and layout of one generation on this rank."""

    plan: HeteroParallelPlan
    schedule: Schedule
    module: object
    opt: Adam
    layout: dict[str, tuple[int, int]]

    def state(self) -> LocalState:
        trainable = self.module.named_state()
        values = {name: p.data for name, p in trainable.items()}
        values.update(self.module.named_buffer_state())
        moments = {kind: {name: self.opt.state[name][kind] for name in trainable} for kind in KINDS[1:]}
        return {"param": values, **moments}

    def load(self, state: LocalState, step_count: int) -> None:
        with torch.no_grad():
            for name, p in self.module.named_state().items():
                p.data.copy_(state["param"][name])
                for kind in KINDS[1:]:
                    self.opt.state[name][kind].copy_(state[kind][name])
            for name, buf in self.module.named_buffer_state().items():
                buf.copy_(state["param"][name])
        self.opt.step_count = step_count


class HeteroBinding:
    def __init__(self, cfg: RefModelConfig, sampler: IndexAddressableSampler, mgr: ResilientCommManager,
                 client: WorkerClient, *, lr: float = 1e-2, use_channels: bool = False, injector=None,
                 timeout: float = 120.0, chunk: int | None = None, checkpointer: SliceCheckpointer | None = None,
                 checkpoint_interval: int = 0, report_timing: bool = True, iter_sleep: float = 0.0):
        self.cfg, self.sampler, self.mgr, self.client = cfg, sampler, mgr, client
        self.lr, self.use_channels, self.injector, self.timeout, self.chunk = lr, use_channels, injector, timeout, chunk
        self.checkpointer, self.checkpoint_interval = checkpointer, checkpoint_interval
        self.report_timing, self.iter_sleep = report_timing, iter_sleep
        self.me = client.worker_id
        self.specs = reference_specs(cfg)
        self.committed: _Generation | None = None
        self.pending: _Generation | None = None
        self.last_transfer: dict = {}

    # ------------------------------------------------------------------ generation build
    def group_specs(self, world: list[str], payload: dict) -> list[GroupSpec]:
        plan = HeteroParallelPlan.from_json(payload["plan"])
        groups = plan.group_specs(reference_partition_sizes(self.cfg))
        if not self.use_channels:
            return groups
        tokens = self.sampler.micro_batch_size * self.cfg.seq_max
        rows = -(-tokens // self.cfg.token_multiple) * self.cfg.token_multiple
        return groups + channel_specs(plan, schedule_from_json(payload["schedule"]), rows)

    def recover(self, comms: GenerationComms, payload: dict, txm: TransactionManager) -> None:
        plan = HeteroParallelPlan.from_json(payload["plan"])
        recovery = payload["recovery"]
        if self.committed is not None and self.me in recovery["local_step"] and txm.has_reduced_grads:
            self.committed.opt.step()  # roll forward: this rank holds the target's reduced gradients
            txm.adopt(recovery["target_iteration"])
        else:
            txm.discard()  # undo the abandoned iteration's buffers before serving as a source
        module = build_stage_module(self.cfg, plan, comms, self.mgr)
        new_holdings = holdings(plan, self.specs, reference_layer_of)
        fresh = _Generation(plan, schedule_from_json(payload["schedule"]), module,
                            Adam(module.named_state(), lr=self.lr), device_layout(new_holdings, self.me))
        if recovery.get("restore"):
            txm.adopt(self._from_checkpoint(fresh))
        elif payload.get("previous_plan") is not None and recovery["target_iteration"] >= 0:
            self._from_peers(fresh, new_holdings, payload, comms)
            txm.adopt(recovery["target_iteration"])
        txm.discard()
        self.pending = fresh

    def _from_peers(self, fresh: _Generation, new_holdings, payload: dict, comms: GenerationComms) -> None:
        recovery = payload["recovery"]
        old_holdings = holdings(HeteroParallelPlan.from_json(payload["previous_plan"]), self.specs,
                                reference_layer_of)
        sources = set(recovery["up_to_date"]) | set(recovery["local_step"])
        moves = plan_transfers(old_holdings, new_holdings, valid_sources=sources, node_of=payload.get("nodes", {}),
                               chunk=self.chunk)
        if moves.lost:
            raise RuntimeError(f"{len(moves.lost)} state slices have no surviving holder")
        serve = self.committed is not None and self.me in sources
        started = time.monotonic()
        state = execute_transfers(moves, self.me, comms, self.mgr, specs=self.specs,
                                  old_layout=device_layout(old_holdings, self.me) if serve else {},
                                  old_state=self.committed.state() if serve else {},
                                  new_layout=fresh.layout, kinds=KINDS, dtype=self.cfg.dtype, device=self.cfg.device,
                                  timeout=self.timeout)
        fresh.load(state, step_count=recovery["target_iteration"] + 1)
        self.last_transfer = dict(transfers=len(moves.transfers), reuse=len(moves.reuse),
                                  received=sum(t.dst == self.me for t in moves.transfers),
                                  seconds=time.monotonic() - started)

    def _from_checkpoint(self, fresh: _Generation) -> int:
        if self.checkpointer is None:
            raise RuntimeError("restore requested but no checkpointer is configured")
        shapes = {key: (spec.global_shape, spec.dim) for key, spec in self.specs.items()}
        iteration = self.checkpointer.latest_complete(shapes)
        if iteration is None:
            raise RuntimeError("no complete checkpoint to restore from")
        state: LocalState = {kind: {} for kind in KINDS}
        for trainable, kinds in ((True, KINDS), (False, KINDS[:1])):
            wanted = [self._slice(key, span) for key, span in fresh.layout.items()
                      if self.specs[key].trainable == trainable]
            for key, per_kind in (self.checkpointer.load(iteration, wanted, kinds=kinds) if wanted else {}).items():
                for kind in kinds:
                    state[kind][key] = per_kind[kind]
        fresh.load(state, step_count=iteration + 1)
        return iteration

    def _slice(self, key: str, span) -> SliceMeta:
        spec = self.specs[key]
        return SliceMeta(key, spec.global_shape, spec.dim, span)

    def build_runtime(self, comms: GenerationComms, payload: dict) -> HeteroRuntime:
        from ..detect.timing import ChunkTimer

        gen = self.pending
        timer = ChunkTimer(use_cuda=False, injector=self.injector) if self.report_timing else None
        return HeteroRuntime(self.cfg, self.sampler, gen.plan, gen.schedule, comms, self.mgr, gen.module,
                             use_channels=self.use_channels, progress=self.client.set_progress,
                             hook=self.injector.on_hook if self.injector is not None else None, timeout=self.timeout,
                             timer=timer, reporter=self.client.report if self.report_timing else None)

    def on_generation_commit(self) -> None:
        self.committed, self.pending = self.pending, None

    # ------------------------------------------------------------------ per iteration
    def buffers(self) -> dict[str, torch.Tensor]:
        return {} if self.committed is None else self.committed.module.transaction_buffers()

    def optimizer_step(self) -> None:
        self.committed.opt.step()

    def discard_grads(self) -> None:
        self.committed.opt.zero_grad()

    def after_commit(self, iteration: int, comms: GenerationComms) -> None:
        if self.iter_sleep:
            time.sleep(self.iter_sleep)
        every = self.checkpoint_interval
        if self.checkpointer is None or not every or (iteration + 1) % every:
            return
        gen = self.committed
        state = gen.state()
        pieces = []
        for key, span in gen.layout.items():
            kinds = KINDS if self.specs[key].trainable else KINDS[:1]
            pieces.append((self._slice(key, span), {kind: state[kind][key] for kind in kinds}))
        self.checkpointer.save(iteration, self.me, pieces, extra={"step_count": gen.opt.step_count}, blocking=True)

    def try_resume(self, txm: TransactionManager) -> None:
        """The hybrid runtime resumes only through the coordinator's ``restore`` recovery."""
