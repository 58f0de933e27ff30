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


def plan_layout(cfg: GPTConfig, *, tp: int, pp: int, dp: int, num_microbatches: int, micro_batch: int, seq_len: int):
    """``(plan, schedule)`` of a ``tp x pp x dp`` layout on one node (device ids ``n0g{i}``)."""
    from ..plan.model_spec import ModelProfile, ModelSpec
    from ..plan.planner import HeteroPlanner, PlannerConfig
    from ..plan.topology import ClusterTopology

    spec = ModelSpec(num_layers=cfg.layers, hidden=cfg.hidden, ffn=cfg.ffn, num_heads=cfg.heads,
                     num_kv_heads=cfg.kv_heads, vocab=cfg.vocab_size, seq_len=seq_len, micro_batch_size=micro_batch)
    pc = PlannerConfig(model=spec, profile=ModelProfile.b200(spec), num_stages=pp, num_replicas=dp, tp=tp,
                       num_microbatches=num_microbatches, sequence_parallel=True, mem_capacity=math.inf)
    planner = HeteroPlanner(pc)
    topo = ClusterTopology.uniform(1, tp * pp * dp)
    plan = planner.initial_plan(topo)
    schedule, _ = planner.schedule(plan, topo)
    return plan, schedule


class GPUHybridTrainer:
    def __init__(self, cfg: GPTConfig, *, tp: int, pp: int, dp: int, global_batch: int, micro_batch: int = 1,
                 seq_len: int | None = None, tp_impl: str = "fused", dp_impl: str = "fused", seed: int = 0,
                 lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0, device=None,
                 data_seed: int = 1):
        from ..comm.comm_manager import ResilientCommManager
        from ..runtime.gpu_executor import TokenSource
        from ..runtime.gpu_runtime import GPUHybridRuntime, gpu_group_specs

        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        if tp * pp * dp != world:
            raise ValueError(f"tp {tp} x pp {pp} x dp {dp} != world size {world}")
        if global_batch % micro_batch:
            raise ValueError("the global batch must be a multiple of the micro-batch")
        self.cfg = cfg
        self.S = seq_len or cfg.seq_len
        self.device = torch.device(device if device is not None else f"cuda:{torch.cuda.current_device()}")
        self.micro_batch = micro_batch
        n_micro = global_batch // micro_batch
        self.plan, self.schedule = plan_layout(cfg, tp=tp, pp=pp, dp=dp, num_microbatches=n_micro,
                                               micro_batch=micro_batch, seq_len=self.S)
        ids = list(self.plan.world)
        self.mgr = ResilientCommManager("nccl" if self.device.type == "cuda" else "gloo", device=str(self.device),
                                        subgroup_mode="local", timeout_s=120)
        specs = gpu_group_specs(self.plan, self.schedule, micro_batch * self.S)
        self.comms = self.mgr.adopt(1, ids, ids[rank], specs)
        self.tokens = TokenSource(cfg.vocab_size, micro_batch, self.S, seed=data_seed)
        self.runtime = GPUHybridRuntime(cfg, self.plan, self.schedule, self.comms, self.mgr, device=self.device,
                                        micro_batch=micro_batch, seq_len=self.S, tokens=self.tokens, tp_impl=tp_impl,
                                        dp_impl=dp_impl, seed=seed, lr=lr, betas=betas, eps=eps,
                                        weight_decay=weight_decay)
        self.tokens_per_step = self.runtime.tokens_per_step
        self.global_batch = global_batch
        self.layout = f"tp{tp}pp{pp}dp{dp}-sp-{tp_impl}tp-{dp_impl}dp"

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

    def close(self) -> None:
        self.runtime.close()
