"""Mixtral-style MoE decoder on this package's kernels, expert parallel over the data-parallel ranks.

Each layer is the Llama attention block followed by a top-k mixture of SwiGLU experts:

    h2 = rmsnorm(x2)
    y  = x2 + sum_k g_k(h2) E_{e_k}(h2)          (route -> dispatch -> experts -> combine)

Dense weights (embedding, attention, norms, router, LM head) are replicated on every rank and
reduced data parallel; expert ``e`` lives on rank ``holder[e]`` only (expert parallelism over
the same ranks, benchmark config 3's EP8 x DP8).  The expert transport is a backend with the
phases of ``parallel.moe_ep.ExpertParallelMoE`` (peer-memory kernels over NVLink) or
``parallel.ep_backend.CollectiveEP`` (``all_to_all``); one routing state is kept per layer
between the forward and the backward of a micro-batch.  The backward through a MoE block needs
the expert-input gradient without the residual path (the experts read ``h2``, the residual is
``x2``): ``grad_pull(residual=False)`` then the MLP norm's backward adds the residual gradient.
(Reference: the MoE block and EP runtime of ``resihp/runtime/moe.py:29-269``, whose GPU model is
Megatron's.)
"""

from __future__ import annotations

import torch

from .. import ops
from .config import GPTConfig
from .params import FlatParams, ParamSpec


def moe_param_specs(cfg: GPTConfig, local_experts: list[int]) -> tuple[list[ParamSpec], list[ParamSpec]]:
    """``(dense, experts)`` specs; ``experts`` holds only ``local_experts``."""
    H, F, E = cfg.hidden, cfg.ffn, cfg.num_experts
    dense = [ParamSpec("embed", (cfg.vocab_size, H))]
    experts: list[ParamSpec] = []
    for l in range(cfg.layers):
        p = f"layers.{l}."
        dense += [ParamSpec(p + "attn_norm", (H,), init="ones"), ParamSpec(p + "wqkv", (cfg.qkv_rows, H)),
                  ParamSpec(p + "wo", (H, cfg.heads * cfg.head_dim)), ParamSpec(p + "mlp_norm", (H,), init="ones"),
                  ParamSpec(p + "router", (E, H))]
        for e in local_experts:
            experts += [ParamSpec(f"{p}experts.{e}.w13", (2 * F, H)), ParamSpec(f"{p}experts.{e}.w2", (H, F))]
    dense += [ParamSpec("final_norm", (H,), init="ones"), ParamSpec("lm_head", (cfg.vocab_size, H))]
    return dense, experts


class MoEModel:
    def __init__(self, cfg: GPTConfig, device, *, ep, holder: list, rank: int, micro_batch: int = 1,
                 seq_len: int | None = None, seed: int = 0, dense_shard: tuple[int, int] = (0, 1),
                 dense_factories=(None, None), init: bool = True):
        """``holder[e]``: the rank of expert ``e`` or the list of its replicas' ranks."""
        if not cfg.is_moe:
            raise ValueError("MoEModel needs a config with experts")
        self.cfg, self.device = cfg, torch.device(device)
        self.ep = ep
        self.seed = seed
        self.holders = [list(h) if isinstance(h, (list, tuple)) else [int(h)] for h in holder]
        self.local = [e for e in range(cfg.num_experts) if rank in self.holders[e]]
        self.mb = micro_batch
        self.S = seq_len or cfg.seq_len
        self.T = self.mb * self.S
        dense, experts = moe_param_specs(cfg, self.local)
        self.dense = FlatParams(dense, self.device, shard_rank=dense_shard[0], shard_count=dense_shard[1],
                                buffer_factory=dense_factories[0], opt_factory=dense_factories[1])
        self.experts = FlatParams(experts, self.device)
        if init:
            self.dense.initialize(seed, cfg.init_std)
            self.experts.initialize(seed, cfg.init_std)
        self.cos, self.sin = ops.rope_tables(self.S, cfg.head_dim, cfg.rope_theta, self.device)
        self._alloc()

    def rebuild_experts(self, holders: list, rank: int, ep) -> None:
        """Switch to a new expert placement: fresh (uninitialised) expert buffers for the experts
        this rank now holds, to be filled with migrated state, and the new transport."""
        self.holders = [list(h) if isinstance(h, (list, tuple)) else [int(h)] for h in holders]
        self.local = [e for e in range(self.cfg.num_experts) if rank in self.holders[e]]
        _, experts = moe_param_specs(self.cfg, self.local)
        self.experts = FlatParams(experts, self.device)
        self.ep = ep

    def _alloc(self) -> None:
        c, T, dev = self.cfg, self.T, self.device
        H, L = c.hidden, c.layers
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.xs = [torch.empty(T, H, **bf) for _ in range(L + 1)]
        self.x2 = [torch.empty(T, H, **bf) for _ in range(L)]
        self.h2 = [torch.empty(T, H, **bf) for _ in range(L)]
        self.qkv = [torch.empty(T, c.qkv_rows, **bf) for _ in range(L)]
        self.o = [torch.empty(T, c.heads * c.head_dim, **bf) for _ in range(L)]
        self.lse = [torch.empty(self.mb, c.heads, self.S, **f32) for _ in range(L)]
        self.rstd1 = [torch.empty(T, **f32) for _ in range(L)]
        self.rstd2 = [torch.empty(T, **f32) for _ in range(L)]
        self.states: list[dict | None] = [None] * L
        self.ws_h = torch.empty(T, H, **bf)
        self.ws_dh = torch.empty(T, H, **bf)
        self.ws_dx = torch.empty(T, H, **bf)
        self.ws_dx2 = torch.empty(T, H, **bf)
        self.ws_do = torch.empty(T, c.heads * c.head_dim, **bf)
        self.ws_dqkv = torch.empty(T, c.qkv_rows, **bf)
        self.hf = torch.empty(T, H, **bf)
        self.rstd_f = torch.empty(T, **f32)
        self.logits = torch.empty(T, c.vocab_size, **bf)
        self.loss_acc = torch.zeros((), **f32)

    # ------------------------------------------------------------------ views
    def expert_weights(self, l: int) -> dict[int, tuple[torch.Tensor, torch.Tensor]]:
        P = self.experts
        return {e: (P.w(f"layers.{l}.experts.{e}.w13"), P.w(f"layers.{l}.experts.{e}.w2")) for e in self.local}

    def expert_grads(self, l: int) -> dict[int, tuple[torch.Tensor, torch.Tensor]]:
        P = self.experts
        return {e: (P.g(f"layers.{l}.experts.{e}.w13"), P.g(f"layers.{l}.experts.{e}.w2")) for e in self.local}

    def _qkv_views(self, i: int):
        c, D = self.cfg, self.cfg.head_dim
        q = self.qkv[i]
        return q[:, : c.heads * D], q[:, c.heads * D:(c.heads + c.kv_heads) * D], q[:, (c.heads + c.kv_heads) * D:]

    def _rms(self, x, w, out, rstd):
        return ops.rmsnorm_fwd(x, w, float(self.cfg.norm_eps), out=out, rstd=rstd)[0]

    # ------------------------------------------------------------------ forward / backward
    def forward_backward(self, ids: torch.Tensor, labels: torch.Tensor, grad_scale: float) -> None:
        """One micro-batch: forward, loss (summed into ``loss_acc``), backward; gradients of both
        parameter sets accumulate."""
        c, P, ep = self.cfg, self.dense, self.ep
        D = c.head_dim
        ops.embedding_fwd(ids, P.w("embed"), out=self.xs[0])
        for i in range(c.layers):
            p = f"layers.{i}."
            x = self.xs[i]
            self._rms(x, P.w(p + "attn_norm"), self.ws_h, self.rstd1[i])
            ops.gemm(self.ws_h, P.w(p + "wqkv"), out=self.qkv[i])
            q, k, v = self._qkv_views(i)
            ops.rope_(q, c.heads, D, self.cos, self.sin, self.S)
            ops.rope_(k, c.kv_heads, D, self.cos, self.sin, self.S)
            ops.attention_fwd(q, k, v, batch=self.mb, seq=self.S, heads=c.heads, kv_heads=c.kv_heads, head_dim=D,
                              out=self.o[i], lse=self.lse[i])
            ops.gemm(self.o[i], P.w(p + "wo"), residual=x, out=self.x2[i])
            self._rms(self.x2[i], P.w(p + "mlp_norm"), self.h2[i], self.rstd2[i])
            ep.route(self.h2[i], P.w(p + "router"))
            ep.exchange_counts()
            ep.dispatch()
            ep.experts_forward(self.expert_weights(i), keep_input=True)
            self.xs[i + 1].copy_(ep.combine(self.x2[i]))
            ep.finish_forward()
            self.states[i] = ep.take_state()
        self._rms(self.xs[-1], P.w("final_norm"), self.hf, self.rstd_f)
        ops.gemm(self.hf, P.w("lm_head"), out=self.logits)
        loss = ops.cross_entropy_(self.logits, labels, grad_scale=grad_scale)
        self.loss_acc += loss.sum()
        # backward
        dx = self.ws_dx
        ops.gemm(self.logits, P.w("lm_head"), b_t=True, out=self.ws_dh)
        ops.gemm(self.logits, self.hf, a_t=True, b_t=True, out=P.g("lm_head"), accumulate=True)
        ops.rmsnorm_bwd(self.xs[-1], P.w("final_norm"), self.rstd_f, self.ws_dh, P.g("final_norm"), out=dx)
        for i in reversed(range(c.layers)):
            p = f"layers.{i}."
            ep.put_state(self.states[i])
            ep.grad_push(dx)
            ep.experts_backward(self.expert_weights(i), self.expert_grads(i))
            ep.grad_pull(P.w(p + "router"), P.g(p + "router"), residual=False, out=self.ws_dh)
            ep.take_state()
            self.states[i] = None
            ops.rmsnorm_bwd(self.x2[i], P.w(p + "mlp_norm"), self.rstd2[i], self.ws_dh, P.g(p + "mlp_norm"), dres=dx,
                            out=self.ws_dx2)
            dx2 = self.ws_dx2
            ops.gemm(dx2, P.w(p + "wo"), b_t=True, out=self.ws_do)
            ops.gemm(dx2, self.o[i], a_t=True, b_t=True, out=P.g(p + "wo"), accumulate=True)
            q, k, v = self._qkv_views(i)
            dq = self.ws_dqkv[:, : c.heads * D]
            dk = self.ws_dqkv[:, c.heads * D:(c.heads + c.kv_heads) * D]
            dv = self.ws_dqkv[:, (c.heads + c.kv_heads) * D:]
            ops.attention_bwd(q, k, v, self.o[i], self.ws_do, self.lse[i], dq, dk, dv, batch=self.mb, seq=self.S,
                              heads=c.heads, kv_heads=c.kv_heads, head_dim=D)
            ops.rope_(dq, c.heads, D, self.cos, self.sin, self.S, inverse=True)
            ops.rope_(dk, c.kv_heads, D, self.cos, self.sin, self.S, inverse=True)
            self._rms(self.xs[i], P.w(p + "attn_norm"), self.ws_h, self.rstd1[i])
            ops.gemm(self.ws_dqkv, P.w(p + "wqkv"), b_t=True, out=self.ws_dh)
            ops.gemm(self.ws_dqkv, self.ws_h, a_t=True, b_t=True, out=P.g(p + "wqkv"), accumulate=True)
            ops.rmsnorm_bwd(self.xs[i], P.w(p + "attn_norm"), self.rstd1[i], self.ws_dh, P.g(p + "attn_norm"),
                            dres=dx2, out=dx)
        ops.embedding_bwd(ids, dx, P.g("embed"))
