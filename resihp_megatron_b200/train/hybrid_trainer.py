"""GPU training engine for hybrid parallelism on one node: TP (+ sequence parallel) x PP x DP.

``GPUHybridTrainer.train_step()`` is the public entry point: it runs one optimizer step of the
global batch (``num_microbatches`` micro-batches of synthetic tokens from ``TokenSource``, copied
from pinned host memory by the ranks that consume them), reads the global mean loss back to the
host and returns it.  ``step_device()`` is the same step without the host read.

The layout comes from the joint planner (``plan.planner.HeteroPlanner``: device placement,
min-max layer partition, micro-batch assignment) and its validated pipeline schedule, exactly as
in the resilient CPU runtime; the launcher's default process group (``torchrun``) is adopted as
generation 1 and the plan's TP, DP and pipeline-channel groups are created on it.
(Reference: the Megatron-Core binding, ``resihp/train/megatron_binding.py``, and the plan-driven
runtime, ``resihp/runtime/hetero_runtime.py``.)
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..models.config import GPTConfig


def ensure_process_group(device: torch.device) -> None:
    """A one-rank process group when no launcher set one up (single GPU), so the runtime's
    collectives have a group to run on."""
    if dist.is_initialized():
        return
    backend = "nccl" if device.type == "cuda" else "gloo"
    kw = {"device_id": device} if device.type == "cuda" else {}
    dist.init_process_group(backend, store=dist.HashStore(), rank=0, world_size=1, **kw)


def layout_planner(cfg: GPTConfig, *, tp: int, pp: int, dp: int, num_microbatches: int, micro_batch: int,
                   seq_len: int, sequence_parallel: bool = True, vpp: int = 1, split_backward: bool = False):
    """The joint planner for a ``tp x pp x dp`` layout of ``cfg`` on one node, and the node's
    topology (device ids ``n0g{i}``).  ``vpp``: model chunks per pipeline slot (interleaved
    schedule); ``split_backward``: zero-bubble schedules with the weight-gradient pass split off."""
    from ..plan.model_spec import ModelProfile, ModelSpec
    from ..plan.planner import HeteroPlanner, PlannerConfig
    from ..plan.topology import ClusterTopology

    spec = ModelSpec(num_layers=cfg.layers, hidden=cfg.hidden, ffn=cfg.ffn, num_heads=cfg.heads,
                     num_kv_heads=cfg.kv_heads, vocab=cfg.vocab_size, seq_len=seq_len, micro_batch_size=micro_batch)
    # the measured profile of this layer shape when one is committed, else the analytic B200 one
    profile = ModelProfile.calibrated(spec) or ModelProfile.b200(spec)
    pc = PlannerConfig(model=spec, profile=profile, num_stages=pp, num_replicas=dp, tp=tp,
                       num_microbatches=num_microbatches, sequence_parallel=sequence_parallel, mem_capacity=math.inf,
                       vpp=vpp, split_backward=split_backward)
    return HeteroPlanner(pc), ClusterTopology.uniform(1, tp * pp * dp)


class GPUHybridTrainer:
    def __init__(self, cfg: GPTConfig, *, tp: int, pp: int, dp: int, global_batch: int, micro_batch: int = 1,
                 seq_len: int | None = None, tp_impl: str = "fused", dp_impl: str = "fused", seed: int = 0,
                 lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0, device=None,
                 data_seed: int = 1, migrate: str = "p2p", fp8=None, sequence_parallel: bool = True,
                 vpp: int = 1, split_backward: bool = False):
        """``migrate``: how a reconfiguration moves state on GPUs -- ``"p2p"`` (one strided peer
        copy launch per rank over NVLink, ``parallel.migration``) or ``"nccl"`` (one send/receive
        per slice and kind, ``state.transfer_engine``).  ``fp8``: an ``Fp8Recipe`` (block-scaled
        fp8 projections; the per-layer amax histories migrate and checkpoint with their layers).
        ``sequence_parallel=False``: plain tensor parallelism (replicated token rows, GEMM ->
        all-reduce).  ``vpp``: model chunks per pipeline slot (interleaved 1F1B);
        ``split_backward``: zero-bubble schedules (the weight-gradient pass of each micro-batch
        runs separately, where the schedule puts it)."""
        from ..comm.comm_manager import ResilientCommManager
        from ..runtime.gpu_executor import TokenSource
        from ..runtime.gpu_runtime import GPUHybridRuntime

        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        if tp * pp * dp != world:
            raise ValueError(f"tp {tp} x pp {pp} x dp {dp} != world size {world}")
        if global_batch % micro_batch:
            raise ValueError("the global batch must be a multiple of the micro-batch")
        if vpp > 1 and pp < 2:
            raise ValueError("interleaving (vpp > 1) needs at least 2 pipeline stages to alternate between")
        if migrate not in ("p2p", "nccl"):
            raise ValueError(migrate)
        self.migrate = migrate
        self.cfg = cfg
        self.S = seq_len or cfg.seq_len
        self.device = torch.device(device if device is not None else f"cuda:{torch.cuda.current_device()}")
        self.micro_batch = micro_batch
        n_micro = global_batch // micro_batch
        self.sequence_parallel = sequence_parallel
        self.planner, self.topology = layout_planner(cfg, tp=tp, pp=pp, dp=dp, num_microbatches=n_micro,
                                                     micro_batch=micro_batch, seq_len=self.S,
                                                     sequence_parallel=sequence_parallel, vpp=vpp,
                                                     split_backward=split_backward)
        self.plan = self.planner.initial_plan(self.topology)
        self.schedule, _ = self.planner.schedule(self.plan, self.topology)
        ids = list(self.plan.world)
        # NCCL: the plan's groups come from one ncclCommSplit per layer of disjoint groups
        # ("split"), not one communicator creation per group; gloo creates them one by one
        self.mgr = ResilientCommManager("nccl" if self.device.type == "cuda" else "gloo", device=str(self.device),
                                        subgroup_mode="split" if self.device.type == "cuda" else "local",
                                        timeout_s=120)
        self.comms = self.mgr.adopt(1, ids, ids[rank], self._group_specs(self.plan, self.schedule))
        self.tokens = TokenSource(cfg.vocab_size, micro_batch, self.S, seed=data_seed)
        self.fp8 = fp8
        self.opts = dict(micro_batch=micro_batch, seq_len=self.S, tokens=self.tokens, tp_impl=tp_impl, dp_impl=dp_impl,
                         seed=seed, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, fp8=fp8)
        self.runtime = GPUHybridRuntime(cfg, self.plan, self.schedule, self.comms, self.mgr, device=self.device,
                                        **self.opts)
        self.tokens_per_step = self.runtime.tokens_per_step
        self.global_batch = global_batch
        self.layout = (f"tp{tp}pp{pp}dp{dp}-{'sp' if sequence_parallel else 'nosp'}-{tp_impl}tp-{dp_impl}dp"
                       + ("-fp8" if fp8 is not None else ""))
        self.last_reconfig: dict | None = None

    def tensor_specs(self):
        """Logical tensors of the job (with the fp8 amax histories when fp8 is on)."""
        from ..runtime.gpu_state import gpu_tensor_specs

        return gpu_tensor_specs(self.cfg, self.fp8.history if self.fp8 is not None else 0)

    def _group_specs(self, plan, schedule):
        from ..runtime.gpu_runtime import gpu_group_specs
        from ..runtime.gpu_state import partition_sizes

        return gpu_group_specs(plan, schedule, self.micro_batch * self.S, partition_sizes(self.cfg))

    def step_device(self) -> torch.Tensor:
        """One step; the global mean loss as a 0-d device tensor (no host synchronisation)."""
        return self.runtime.run_iteration()

    def train_step(self) -> float:
        """One step through the public path: the micro-batches' tokens are copied from pinned host
        memory by the ranks that consume them, and the loss is read back to the host."""
        value = float(self.step_device().item())
        self.runtime.check()
        return value

    @property
    def h2d_bytes_last_step(self) -> int:
        return self.runtime.executor.h2d_bytes

    def check(self) -> None:
        self.runtime.check()

    # ------------------------------------------------------------------ checkpoints (T2)
    def save_checkpoint(self, directory) -> int:
        """Write this rank's slices of the last completed step to ``directory`` in the shared
        slice-checkpoint format (every rank calls it; collective inside ZeRO data-parallel
        groups).  Returns the checkpoint's iteration."""
        from ..runtime.gpu_state import checkpoint_slices
        from ..state.checkpoint import SliceCheckpointer

        it = self.runtime.iteration - 1
        me = self.plan.world[self.comms.rank]
        ck = SliceCheckpointer(directory)
        ck.save(it, me, checkpoint_slices(self.runtime, self.tensor_specs()),
                extra={"step_count": self.runtime.step_count, "layout": self.layout}, blocking=True)
        return it

    def load_checkpoint(self, directory, iteration: int | None = None) -> int:
        """Load the newest complete checkpoint (or ``iteration``) from ``directory``, whatever
        layout wrote it, and continue from the step after it."""
        from ..runtime.gpu_state import load_checkpoint_into
        from ..state.checkpoint import SliceCheckpointer

        specs = self.tensor_specs()
        ck = SliceCheckpointer(directory)
        if iteration is None:
            iteration = ck.latest_complete({k: (s.global_shape, s.dim) for k, s in specs.items()})
            if iteration is None:
                raise FileNotFoundError(f"no complete checkpoint under {directory}")
        load_checkpoint_into(self.runtime, ck, iteration, specs)
        self.runtime.iteration = iteration + 1
        return iteration

    # ------------------------------------------------------------------ live reconfiguration
    def reconfigure(self, leaving: list[int], *, store=None, store_addr=None, store_prefix: str | None = None) -> bool:
        """Planned removal of the ranks ``leaving`` (e.g. a GPU evicted as fail-slow), between
        steps; every current rank calls it.  Each rank first exports its slot's full
        tensor-parallel-local state (ZeRO shards all-gathered inside each data-parallel group),
        so every interval of every tensor is also held by a surviving replica; the planner
        re-plans on the remaining devices (TP shrink of the weakened group or its eviction with
        micro-batch migration, min-max layer repartition); the survivors rebuild the
        communicators without the leavers (NCCL shrink, or a fresh world on ``store`` /
        ``store_addr``), build the new generation's runtime and pull every slice of parameters
        and Adam moments they now hold from the old holders (``state.transfer_plan`` /
        ``state.transfer_engine``); the global batch, data order and step count are unchanged.
        Returns False on a rank that leaves or becomes standby (it must not use the trainer
        afterwards).  Phase timings land in ``last_reconfig``.  (Reference: the worker's
        generation build and state migration, ``resihp/train/resilient_loop.py:113-160`` and
        ``resihp/train/hetero_binding.py:95-130``.)"""
        import time

        from ..runtime.gpu_state import export_state

        marks = [("start", time.perf_counter())]

        def mark(name: str) -> None:
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            marks.append((name, time.perf_counter()))

        rt, old_plan = self.runtime, self.plan
        me = old_plan.world[self.comms.rank]
        state, layout = export_state(rt)
        step, iteration = rt.step_count, rt.iteration
        mark("export")
        gone = {old_plan.world[r] for r in leaving}
        topo = self.topology.without(sorted(gone))
        new_plan = self.planner.replan(old_plan, topo)
        new_schedule, _ = self.planner.schedule(new_plan, topo)
        active = {d for g in new_plan.stage_groups for d in g.devices}
        mark("plan")
        if me not in active:
            rt.close()
            self.runtime = None
            return False
        new_world = [d for d in new_plan.world if d in active]
        if list(new_plan.world) != new_world:  # standby devices leave the job as well
            new_plan = _without_standby(new_plan, new_world)
            new_schedule, _ = self.planner.schedule(new_plan, topo)
        comms = self.mgr.build(new_plan.generation, new_world, me, self._group_specs(new_plan, new_schedule),
                               store=store, store_addr=store_addr, store_prefix=store_prefix)
        mark("regroup")
        self._migrate_to(old_plan, new_plan, new_schedule, comms, me, new_world, state, layout, step, iteration, mark)
        self.last_reconfig = {name: round(t - marks[i][1], 4) for i, (name, t) in enumerate(marks[1:])}
        self.last_reconfig.update(self._moved, layout=[(g.replica, g.stage, g.tp, list(g.layers))
                                                       for g in new_plan.stage_groups], world=len(new_world),
                                  regroup_phases=comms.stats.get("phases_s"), regroup_path=comms.path)
        return True

    def reshard(self, tp: int, pp: int, dp: int) -> None:
        """Planned live change of the layout on the same GPUs between steps (e.g. TP4 x DP2 ->
        TP2 x DP4): every rank exports its slot's state, the joint planner lays out the new
        degrees, the plan's groups are created on the existing world, and parameters, Adam
        moments and the fp8 amax histories move slice by slice into the new layout (peer copies
        over NVLink on GPUs); global batch, data order and step count are unchanged.  Phase
        timings land in ``last_reconfig``."""
        import dataclasses
        import time

        from ..runtime.gpu_state import export_state

        marks = [("start", time.perf_counter())]

        def mark(name: str) -> None:
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            marks.append((name, time.perf_counter()))

        rt, old_plan = self.runtime, self.plan
        world = list(old_plan.world)
        if tp * pp * dp != len(world):
            raise ValueError(f"tp {tp} x pp {pp} x dp {dp} != {len(world)} GPUs")
        me = world[self.comms.rank]
        state, layout = export_state(rt)
        step, iteration = rt.step_count, rt.iteration
        mark("export")
        planner, topo = layout_planner(self.cfg, tp=tp, pp=pp, dp=dp, num_microbatches=old_plan.num_microbatches,
                                       micro_batch=self.micro_batch, seq_len=self.S,
                                       sequence_parallel=self.sequence_parallel)
        new_plan = dataclasses.replace(planner.initial_plan(topo), generation=old_plan.generation + 1)
        if list(new_plan.world) != world:
            raise RuntimeError("the new layout names other devices than the current world")
        new_schedule, _ = planner.schedule(new_plan, topo)
        mark("plan")
        comms = self.mgr.adopt(new_plan.generation, world, me, self._group_specs(new_plan, new_schedule))
        mark("regroup")
        self._migrate_to(old_plan, new_plan, new_schedule, comms, me, world, state, layout, step, iteration, mark)
        self.planner, self.topology = planner, topo
        self.layout = f"tp{tp}pp{pp}dp{dp}-" + self.layout.split("-", 1)[1]
        self.last_reconfig = {name: round(t - marks[i][1], 4) for i, (name, t) in enumerate(marks[1:])}
        self.last_reconfig.update(self._moved, layout=[(g.replica, g.stage, g.tp, list(g.layers))
                                                       for g in new_plan.stage_groups], world=len(world))

    def _migrate_to(self, old_plan, new_plan, new_schedule, comms, me, new_world, state, layout, step, iteration,
                    mark) -> None:
        """Build the new generation's runtime, move every slice it needs from the old holders
        and switch to it (the old runtime is closed)."""
        from ..runtime.gpu_runtime import GPUHybridRuntime
        from ..runtime.gpu_state import KINDS, gpu_layer_of, import_state
        from ..state.layer_registry import device_layout, holdings
        from ..state.transfer_engine import execute_transfers
        from ..state.transfer_plan import plan_transfers

        rt = self.runtime
        new_rt = GPUHybridRuntime(self.cfg, new_plan, new_schedule, comms, self.mgr, device=self.device, init=False,
                                  **self.opts)
        mark("build")
        specs = self.tensor_specs()
        layer_of = gpu_layer_of(self.cfg.layers)
        new_h = holdings(new_plan, specs, layer_of)
        tplan = plan_transfers(holdings(old_plan, specs, layer_of), new_h, valid_sources=set(new_world),
                               node_of={d: "n0" for d in old_plan.world})
        if tplan.lost:
            raise RuntimeError(f"{len(tplan.lost)} state slices have no surviving holder")
        new_layout = device_layout(new_h, me)
        if self.device.type == "cuda" and self.migrate == "p2p":
            from ..parallel.migration import migrate_p2p
            from ..parallel.symm import exchange_via_group

            new_state = {k: {key: torch.empty(specs[key].local_shape(iv), dtype=torch.float32, device=self.device)
                             for key, iv in new_layout.items()} for k in KINDS}
            migrate_p2p(tplan, me, new_world, specs=specs, old_h=holdings(old_plan, specs, layer_of), new_h=new_h,
                        old_state=state, new_state=new_state, kinds=KINDS, device=self.device,
                        exchange=exchange_via_group(None), abort=new_rt.abort)
        else:
            new_state = execute_transfers(tplan, me, comms, self.mgr, specs=specs, old_layout=layout,
                                          old_state=state, new_layout=new_layout, kinds=KINDS, dtype=torch.float32,
                                          device=str(self.device))
        import_state(new_rt, new_state, step)
        new_rt.iteration = iteration
        moved = sum(t.numel() * t.element_size() for k in KINDS for key, t in new_state[k].items()
                    if k == KINDS[0] or specs[key].trainable)
        del new_state, state
        mark("migrate")
        rt.close()
        self.runtime, self.plan, self.schedule, self.comms = new_rt, new_plan, new_schedule, comms
        mark("commit")
        self._moved = {"bytes_loaded": moved, "transfers": len(tplan.transfers)}

    def close(self) -> None:
        if self.runtime is not None:
            self.runtime.close()
            self.runtime = None


def _without_standby(plan, world: list[str]):
    """The same plan over a world without its standby devices."""
    from dataclasses import replace

    return replace(plan, world=tuple(world), standby=())
