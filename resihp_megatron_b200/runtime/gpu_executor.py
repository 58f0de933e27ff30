"""GPU stage executor for the pipeline IR interpreter: the Llama stages of ``models.tp_stage``.

``Interpreter`` (``runtime/interpreter.py``) walks this slot's instruction stream and calls
``forward`` / ``backward`` per micro-batch; the executor feeds the stage its token rows (first
stage) or the activation received over the pipeline boundary, and the labels (last stage).

Data: micro-batch ``mb`` of iteration ``it`` is ``micro_batch`` sequences of uniform random
token ids from a generator seeded by ``(seed, it, mb)`` -- a function of the global micro-batch
index only, so any layout, any replica that executes the micro-batch, and a replay after a
reconfiguration see the same tokens (the reference's index-addressable sampler,
``resihp/state/rng_data.py:41``).  The host draws them into pinned memory and each rank copies
its sequence-parallel rows to the device asynchronously.
"""

from __future__ import annotations

import torch

from ..comm.p2p import local_rows
from ..plan.hetero_plan import HeteroParallelPlan


class TokenSource:
    def __init__(self, vocab: int, micro_batch: int, seq_len: int, seed: int = 1, pin: bool = True):
        self.vocab, self.micro_batch, self.seq_len, self.seed = vocab, micro_batch, seq_len, seed
        self.pin = pin and torch.cuda.is_available()

    def tokens(self, iteration: int, mb: int) -> tuple[torch.Tensor, torch.Tensor]:
        """``(ids, labels)``, each ``[micro_batch * seq_len]`` int64 on the host."""
        g = torch.Generator().manual_seed((self.seed * 1_000_003 + iteration) * 1_000_003 + mb)
        seq = torch.randint(0, self.vocab, (self.micro_batch, self.seq_len + 1), generator=g)
        ids, labels = seq[:, :-1].reshape(-1), seq[:, 1:].reshape(-1)
        if self.pin:
            ids, labels = ids.pin_memory(), labels.pin_memory()
        return ids, labels

    def bytes_per_microbatch(self) -> int:
        return 2 * self.micro_batch * self.seq_len * 8


class GPUStageExecutor:
    """``StageExecutor`` of one physical slot running one ``TPStage`` per model chunk (virtual
    stage); a plan without interleaving has one chunk."""

    def __init__(self, stages: dict, plan: HeteroParallelPlan, replica: int, rank: int, tokens: TokenSource,
                 grad_scale: float, sp: bool = True):
        """``sp=False`` (plain TP): every TP rank takes every token row, and only the slot's first
        TP rank counts the loss (the others compute the same value)."""
        self.models = dict(stages)
        self.plan = plan
        self.group = plan.group(replica, min(self.models))
        if self.group.cp != 1:
            raise NotImplementedError("context parallelism is not wired into the GPU stage")
        self.ranks = plan.ranks(self.group)
        self.rank = rank
        self.tokens = tokens
        self.grad_scale = grad_scale
        self.iteration = -1
        first = next(iter(self.models.values()))
        self.device = first.device
        self.T = first.T
        self.sp = sp
        self.rows = local_rows(first.T, self.ranks, rank) if sp else (0, first.T)
        self.counts_loss = sp or self.ranks.index(rank) == 0
        self._host: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.h2d_bytes = 0
        self.split_backward = False  # zero-bubble schedules: weight gradients in the W pass

    def begin_iteration(self, iteration: int) -> None:
        self.iteration = iteration
        self._host.clear()
        for m in self.models.values():
            m.loss_acc.zero_()
        self.h2d_bytes = 0

    def n_rows(self, mb: int) -> int:
        return self.T

    def _device_rows(self, mb: int, which: int) -> torch.Tensor:
        if mb not in self._host:
            self._host[mb] = self.tokens.tokens(self.iteration, mb)  # kept alive until the copy is done
        a, b = self.rows
        host = self._host[mb][which][a:b]
        self.h2d_bytes += host.numel() * host.element_size()
        return host.to(self.device, non_blocking=True)

    def forward(self, mb: int, inp: torch.Tensor | None, stage: int) -> torch.Tensor | None:
        m = self.models[stage]
        ids = self._device_rows(mb, 0) if m.first else None
        labels = self._device_rows(mb, 1) if m.last else None
        return m.forward((stage, mb), ids_local=ids, x_in=inp, labels_local=labels, grad_scale=self.grad_scale)

    def backward(self, mb: int, grad: torch.Tensor | None, stage: int) -> torch.Tensor | None:
        dx = self.models[stage].backward((stage, mb), grad, defer_w=self.split_backward)
        # the stage reuses its gradient workspace; the boundary send gets its own copy
        return None if dx is None else dx.clone()

    def weight_backward(self, mb: int, stage: int) -> None:
        self.models[stage].weight_backward((stage, mb))

    @property
    def loss_sum(self) -> torch.Tensor:
        total = None
        for m in self.models.values():
            if m.last:
                total = m.loss_acc if total is None else total + m.loss_acc
        if total is None or not self.counts_loss:
            total = torch.zeros((), dtype=torch.float32, device=self.device)  # no chunk here counts the loss
        return total
