"""GPU training engine for Mixtral-style MoE models: data parallel dense weights, expert parallel
experts over the same ranks (EP8 x DP8, TP1).

``GPUMoETrainer.train_step()`` runs one optimizer step of the global batch: rank ``r`` takes the
micro-batches ``[r * n, (r + 1) * n)`` of the step (synthetic tokens from ``TokenSource``, copied
from pinned host memory), runs every micro-batch forward and backward with the expert transport
(``ep_impl="peer"``: peer-memory kernels over NVLink; ``"collective"``: ``all_to_all``), reduces
the dense gradients data parallel (``dp_impl="fused"``: the fused peer-memory reduction + Adam +
gather; ``"collective"``: NCCL) and applies Adam to its dense shard and to its own experts (one
holder per expert: no expert reduction).  Returns the global mean token loss.
(Reference: the EP runtime, ``resihp/runtime/moe.py:149-269``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.config import GPTConfig


class GPUMoETrainer:
    def __init__(self, cfg: GPTConfig, *, global_batch: int, micro_batch: int = 1, seq_len: int | None = None,
                 ep_impl: str = "peer", dp_impl: str = "fused", seed: int = 0, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.0, device=None, data_seed: int = 1,
                 holder: list[int] | None = None):
        from ..models.moe_model import MoEModel
        from ..runtime.gpu_executor import TokenSource
        from ..runtime.gpu_runtime import ParamSetSync

        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        if global_batch % (micro_batch * self.world):
            raise ValueError("the global batch must split into whole micro-batches on every rank")
        self.cfg = cfg
        self.S = seq_len or cfg.seq_len
        self.device = torch.device(device if device is not None else f"cuda:{torch.cuda.current_device()}")
        self.micro_batch = micro_batch
        self.n_local = global_batch // (micro_batch * self.world)
        self.global_batch = global_batch
        self.tokens_per_step = global_batch * self.S
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        E = cfg.num_experts
        self.holder = list(holder) if holder is not None else [e * self.world // E for e in range(E)]
        T = micro_batch * self.S
        self.abort = None
        if ep_impl == "peer":
            from ..parallel.moe_ep import ExpertParallelMoE
            from ..parallel.symm import AbortWord, exchange_via_group

            self.abort = AbortWord()
            self.ep = ExpertParallelMoE(self.rank, self.world, exchange_via_group(None), self.device, hidden=cfg.hidden,
                                        num_experts=E, top_k=cfg.top_k, max_tokens=T, holder=self.holder,
                                        abort=self.abort)
        elif ep_impl == "collective":
            from ..parallel.ep_backend import CollectiveEP

            self.ep = CollectiveEP(self.rank, self.world, None, self.device, hidden=cfg.hidden, num_experts=E,
                                   top_k=cfg.top_k, holder=self.holder)
        else:
            raise ValueError(ep_impl)
        ranks = tuple(range(self.world))
        self.dense_sync = ParamSetSync(ranks, self.rank, None, dp_impl, self.device, abort=self.abort)
        self.model = MoEModel(cfg, self.device, ep=self.ep, holder=self.holder, rank=self.rank,
                              micro_batch=micro_batch, seq_len=self.S, seed=seed, dense_shard=self.dense_sync.shard,
                              dense_factories=self.dense_sync.factories)
        self.dense_sync.attach(self.model.dense)
        self.expert_sync = ParamSetSync((self.rank,), self.rank, None, "collective", self.device)
        self.expert_sync.attach(self.model.experts)
        self.tokens = TokenSource(cfg.vocab_size, micro_batch, self.S, seed=data_seed)
        self.iteration = 0
        self.h2d_bytes = 0
        self.layout = f"ep{self.world}dp{self.world}-{ep_impl}ep-{dp_impl}dp"

    def step_device(self) -> torch.Tensor:
        """One step; the global mean loss as a 0-d device tensor (no host synchronisation)."""
        m = self.model
        m.loss_acc.zero_()
        scale = 1.0 / self.tokens_per_step
        self.h2d_bytes = 0
        keep = []
        for j in range(self.n_local):
            ids, labels = self.tokens.tokens(self.iteration, self.rank * self.n_local + j)
            keep.append((ids, labels))  # pinned sources stay alive until their copies ran
            self.h2d_bytes += ids.numel() * ids.element_size() + labels.numel() * labels.element_size()
            m.forward_backward(ids.to(self.device, non_blocking=True), labels.to(self.device, non_blocking=True),
                               scale)
        kw = dict(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.wd)
        self.dense_sync.step(**kw)
        self.expert_sync.step(**kw)
        loss = m.loss_acc.clone()
        if self.world > 1:
            dist.all_reduce(loss)
        self.iteration += 1
        return loss / self.tokens_per_step

    @property
    def h2d_bytes_last_step(self) -> int:
        return self.h2d_bytes

    def train_step(self) -> float:
        value = float(self.step_device().item())
        self.check()
        return value

    def check(self) -> None:
        self.dense_sync.check()
        heap = getattr(self.ep, "heap", None)
        if heap is not None:
            heap.check()

    def close(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.dense_sync.close()
        self.ep.close()
        if self.abort is not None:
            self.abort.close()
            self.abort = None
