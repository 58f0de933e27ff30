"""Llama-style decoder on this package's sm_100a kernels: explicit forward and backward.

The model is functional: weights live in a ``FlatParams`` (bf16 compute copy + fp32 master,
gradient and Adam moments), activations in buffers allocated once for one micro-batch, and
``forward_backward`` runs one micro-batch and accumulates fp32 gradients.  No autograd, no
``nn.Module`` and no allocation inside a step, so a step is a fixed sequence of kernel
launches (capturable in a CUDA graph).

Per layer (``T`` tokens of one micro-batch):

    h   = rmsnorm(x)                 qkv = h Wqkv^T          rope(q, k)
    o   = attention(q, k, v)         x2  = x + o Wo^T        (residual fused in the GEMM epilogue)
    h2  = rmsnorm(x2)                gu  = h2 W13^T          a = silu(gate) * up
    x'  = x2 + a W2^T

With ``cfg.mlp == "gelu"`` (the GPT MLP) the input projection is ``w1`` alone and
``a = gelu(h2 W1^T)``.  With an ``Fp8Recipe`` the four projections of every layer run as
block-scaled fp8 GEMMs (``models.fp8_linear``); the LM head stays bf16.

Saved for backward: x, x2, qkv (after RoPE), o, lse, gu and the two rstd vectors; h, h2 and
``a`` are recomputed (cheap, bandwidth bound), which keeps activations at ~23 bytes x hidden
per token per layer.  Gradients of every GEMM use the MN-major operand modes of the GEMM
kernel, so no transpose is materialised.

The reference framework delegates the GPU model to Megatron-Core
(``resihp/runtime/megatron_runtime.py:162``); its CPU semantics oracle is
``resihp/runtime/reference_model.py``.
"""

from __future__ import annotations

import torch

from .. import ops
from .config import GPTConfig
from .params import FlatParams, ParamSpec


def layer_param_specs(cfg: GPTConfig, layer: int, tp_rank: int = 0, tp_size: int = 1) -> list[ParamSpec]:
    """Parameters of one decoder layer (column-parallel qkv / w13, row-parallel wo / w2)."""
    from ..utils.intervals import even_split

    H, D, F = cfg.hidden, cfg.head_dim, cfg.ffn
    qh = even_split(cfg.heads, tp_size)[tp_rank]
    kh = even_split(cfg.kv_heads, tp_size)[tp_rank]
    fr = even_split(F, tp_size)[tp_rank]
    nq, nk, nf = qh[1] - qh[0], kh[1] - kh[0], fr[1] - fr[0]
    p = f"layers.{layer}."
    if tp_size == 1:
        return [
            ParamSpec(p + "attn_norm", (H,), init="ones"),
            ParamSpec(p + "wqkv", ((cfg.heads + 2 * cfg.kv_heads) * D, H)),
            ParamSpec(p + "wo", (H, cfg.heads * D)),
            ParamSpec(p + "mlp_norm", (H,), init="ones"),
            ParamSpec(p + fc1_name(cfg), (cfg.mlp_in, H)),
            ParamSpec(p + "w2", (H, F)),
        ]
    # Sharded: q/k/v and gate/up are stored as separate logical tensors so each rank's slice
    # is a contiguous row range of every logical tensor.
    return [
        ParamSpec(p + "attn_norm", (H,), init="ones"),
        ParamSpec(p + "wq", (nq * D, H), (cfg.heads * D, H), 0, (qh[0] * D, qh[1] * D)),
        ParamSpec(p + "wk", (nk * D, H), (cfg.kv_heads * D, H), 0, (kh[0] * D, kh[1] * D)),
        ParamSpec(p + "wv", (nk * D, H), (cfg.kv_heads * D, H), 0, (kh[0] * D, kh[1] * D)),
        ParamSpec(p + "wo", (H, nq * D), (H, cfg.heads * D), 1, (qh[0] * D, qh[1] * D)),
        ParamSpec(p + "mlp_norm", (H,), init="ones"),
        ParamSpec(p + "w1", (nf, H), (F, H), 0, fr),
    ] + ([ParamSpec(p + "w3", (nf, H), (F, H), 0, fr)] if cfg.gated else []) + [
        ParamSpec(p + "w2", (H, nf), (H, F), 1, fr),
    ]


def fc1_name(cfg: GPTConfig) -> str:
    """The MLP's input projection in the unsharded layout: ``w13 = [w1; w3]`` (SwiGLU) or ``w1``."""
    return "w13" if cfg.gated else "w1"


def mlp_act_fwd(cfg: GPTConfig, gu: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    return ops.swiglu_fwd(gu, out=out) if cfg.gated else ops.gelu_fwd(gu, out=out)


def mlp_act_bwd(cfg: GPTConfig, gu: torch.Tensor, da: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    return ops.swiglu_bwd(gu, da, out=out) if cfg.gated else ops.gelu_bwd(gu, da, out=out)


def model_param_specs(cfg: GPTConfig, layers: range | None = None, first: bool = True, last: bool = True):
    specs: list[ParamSpec] = []
    if first:
        specs.append(ParamSpec("embed", (cfg.vocab_size, cfg.hidden)))
    for l in (layers if layers is not None else range(cfg.layers)):
        specs.extend(layer_param_specs(cfg, l))
    if last:
        specs.append(ParamSpec("final_norm", (cfg.hidden,), init="ones"))
        specs.append(ParamSpec("lm_head", (cfg.vocab_size, cfg.hidden)))
    return specs


class LlamaModel:
    """Single-device Llama decoder (optionally a contiguous layer range of it, for pipelines)."""

    def __init__(self, cfg: GPTConfig, device="cuda", *, micro_batch: int = 1, seq_len: int | None = None,
                 seed: int = 0, layers: range | None = None, first: bool = True, last: bool = True,
                 shard_rank: int = 0, shard_count: int = 1, buffer_factory=None, opt_factory=None, fp8=None):
        """``fp8``: an ``Fp8Recipe`` to run the four linear layers of every decoder layer in
        block-scaled fp8 (the LM head stays bf16)."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.mb = micro_batch
        self.S = seq_len or cfg.seq_len
        self.T = self.mb * self.S
        self.layer_ids = list(layers if layers is not None else range(cfg.layers))
        self.first, self.last = first, last
        self.param_specs = model_param_specs(cfg, self.layer_ids, first, last)
        self.params = FlatParams(self.param_specs, self.device, shard_rank=shard_rank, shard_count=shard_count,
                                 buffer_factory=buffer_factory, opt_factory=opt_factory)
        self.params.initialize(seed, cfg.init_std)
        self.cos, self.sin = ops.rope_tables(self.S, cfg.head_dim, cfg.rope_theta, self.device)
        self.fc1 = fc1_name(cfg)
        self.f8 = None
        if fp8 is not None:
            from .fp8_linear import Fp8Linears, check_shapes

            check_shapes(cfg, self.T)
            self.f8 = Fp8Linears(self.layer_ids, self.device, fp8)
        self._alloc()

    # ------------------------------------------------------------------ buffers
    def release_buffers(self) -> None:
        """Free the activation buffers (a reconfiguration needs the memory)."""
        for name in [k for k, v in vars(self).items() if isinstance(v, (torch.Tensor, list)) and k not in (
                "layer_ids", "param_specs", "cos", "sin")]:
            delattr(self, name)
        torch.cuda.empty_cache()

    def restore_buffers(self, micro_batch: int) -> None:
        """Re-allocate the activation buffers, possibly for another micro-batch size."""
        self.mb = micro_batch
        self.T = self.mb * self.S
        self._alloc()

    def _alloc(self) -> None:
        cfg, T, dev = self.cfg, self.T, self.device
        H, F, V = cfg.hidden, cfg.ffn, cfg.vocab_size
        L = len(self.layer_ids)
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.xs = [torch.empty(T, H, **bf) for _ in range(L + 1)]
        self.x2 = [torch.empty(T, H, **bf) for _ in range(L)]
        self.qkv = [torch.empty(T, cfg.qkv_rows, **bf) for _ in range(L)]
        self.o = [torch.empty(T, cfg.heads * cfg.head_dim, **bf) for _ in range(L)]
        self.lse = [torch.empty(self.mb, cfg.heads, self.S, **f32) for _ in range(L)]
        self.gu = [torch.empty(T, cfg.mlp_in, **bf) for _ in range(L)]
        self.rstd1 = [torch.empty(T, **f32) for _ in range(L)]
        self.rstd2 = [torch.empty(T, **f32) for _ in range(L)]
        self.ws_h = torch.empty(T, H, **bf)
        self.ws_a = torch.empty(T, F, **bf)
        self.ws_da = torch.empty(T, F, **bf)
        self.ws_dh = torch.empty(T, H, **bf)
        self.ws_dx = torch.empty(T, H, **bf)
        self.ws_dx2 = torch.empty(T, H, **bf)
        self.ws_do = torch.empty(T, cfg.heads * cfg.head_dim, **bf)
        self.ws_dqkv = torch.empty(T, cfg.qkv_rows, **bf)
        if self.last:
            self.hf = torch.empty(T, H, **bf)
            self.rstd_f = torch.empty(T, **f32)
            self.logits = torch.empty(T, V, **bf)
        self.loss_acc = torch.zeros((), **f32)

    def activation_bytes(self) -> int:
        tot = 0
        for name, v in vars(self).items():
            if isinstance(v, torch.Tensor) and name not in ("cos", "sin"):
                tot += v.numel() * v.element_size()
            elif isinstance(v, list) and v and isinstance(v[0], torch.Tensor):
                tot += sum(t.numel() * t.element_size() for t in v)
        return tot

    # ------------------------------------------------------------------ helpers
    def _views(self, i: int):
        cfg = self.cfg
        D = cfg.head_dim
        q = self.qkv[i][:, : cfg.heads * D]
        k = self.qkv[i][:, cfg.heads * D: (cfg.heads + cfg.kv_heads) * D]
        v = self.qkv[i][:, (cfg.heads + cfg.kv_heads) * D:]
        return q, k, v

    def _attn_kw(self):
        c = self.cfg
        return dict(batch=self.mb, seq=self.S, heads=c.heads, kv_heads=c.kv_heads, head_dim=c.head_dim)

    # ------------------------------------------------------------------ forward
    def forward(self, ids: torch.Tensor | None = None, x_in: torch.Tensor | None = None) -> torch.Tensor:
        """Run the layers; returns the last residual stream ([T, H] bf16)."""
        cfg, P = self.cfg, self.params
        if self.first:
            ops.embedding_fwd(ids, P.w("embed"), out=self.xs[0])
        else:
            self.xs[0].copy_(x_in)
        if self.f8 is not None:
            self.refresh_fp8_weights()
        for i, l in enumerate(self.layer_ids):
            p = f"layers.{l}."
            x = self.xs[i]
            self._norm_linear(l, "qkv", x, P.w(p + "attn_norm"), self.rstd1[i], P.w(p + "wqkv"), self.qkv[i])
            q, k, v = self._views(i)
            ops.rope_(q, cfg.heads, cfg.head_dim, self.cos, self.sin, self.S)
            ops.rope_(k, cfg.kv_heads, cfg.head_dim, self.cos, self.sin, self.S)
            self._attention_fwd(i, q, k, v)
            self._linear(l, "o", self.o[i], P.w(p + "wo"), self.x2[i], residual=x)
            self._norm_linear(l, "fc1", self.x2[i], P.w(p + "mlp_norm"), self.rstd2[i], P.w(p + self.fc1),
                              self.gu[i])
            if self.f8 is not None:  # activation written as the fp8 operand directly
                from ..ops import fp8

                aq = self.f8.act_quant_x(l, "fc2", self.gu[i], cfg.gated)
                fp8.gemm(aq.rowwise(), self.f8.weight(l, "fc2").rowwise(), out=self.xs[i + 1], residual=self.x2[i])
            else:
                mlp_act_fwd(cfg, self.gu[i], self.ws_a)
                self._linear(l, "fc2", self.ws_a, P.w(p + "w2"), self.xs[i + 1], residual=self.x2[i])
        return self.xs[-1]

    # ------------------------------------------------------------------ linear layers (bf16 or fp8)
    def refresh_fp8_weights(self) -> None:
        """Quantise the weights once per optimizer step (before the first forward after it)."""
        P = self.params
        ws = {}
        for l in self.layer_ids:
            p = f"layers.{l}."
            for lin, name in (("qkv", "wqkv"), ("o", "wo"), ("fc1", self.fc1), ("fc2", "w2")):
                ws[(l, lin)] = P.w(p + name)
        self.f8.refresh_weights(ws, P.step)

    def _norm_linear(self, layer, lin, x, norm_w, rstd, w, out):
        """``rmsnorm(x) @ w^T``; fp8: the norm writes the quantised operand directly."""
        if self.f8 is not None:
            from ..ops import fp8

            xq = self.f8.norm_quant_x(layer, lin, x, norm_w, float(self.cfg.norm_eps), rstd)
            return fp8.gemm(xq.rowwise(), self.f8.weight(layer, lin).rowwise(), out=out)
        h, _ = self._rmsnorm(x, norm_w, self.ws_h, rstd)
        return ops.gemm(h, w, out=out)

    def _linear(self, layer, lin, x, w, out, residual=None):
        if self.f8 is not None:
            return self.f8.forward(layer, lin, x, out, residual=residual)
        return ops.gemm(x, w, out=out, residual=residual)

    def _linear_bwd(self, layer, lin, dy, x, w, dx_out, grad):
        """dgrad into ``dx_out``, wgrad accumulated into ``grad``."""
        if self.f8 is not None:
            return self.f8.backward(layer, lin, dy, x, dx_out, grad)
        ops.gemm(dy, w, b_t=True, out=dx_out)
        ops.gemm(dy, x, a_t=True, b_t=True, out=grad, accumulate=True)
        return dx_out

    def _rmsnorm(self, x, w, out, rstd):
        return ops.rmsnorm_fwd(x, w, float(self.cfg.norm_eps), out=out, rstd=rstd)

    def _attention_fwd(self, i, q, k, v):
        ops.attention_fwd(q, k, v, batch=self.mb, seq=self.S, heads=self.cfg.heads, kv_heads=self.cfg.kv_heads,
                          head_dim=self.cfg.head_dim, out=self.o[i], lse=self.lse[i])

    def head_loss(self, labels: torch.Tensor, grad_scale: float) -> torch.Tensor:
        """Final norm + LM head + cross-entropy; leaves dlogits in ``self.logits``."""
        P = self.params
        self._rmsnorm(self.xs[-1], P.w("final_norm"), self.hf, self.rstd_f)
        ops.gemm(self.hf, P.w("lm_head"), out=self.logits)
        loss = ops.cross_entropy_(self.logits, labels, grad_scale=grad_scale)
        return loss

    # ------------------------------------------------------------------ backward
    def backward(self, ids: torch.Tensor | None = None, dx_top: torch.Tensor | None = None) -> torch.Tensor:
        """Backward of the layers given dlogits (last stage) or ``dx_top`` (earlier stages);
        returns the gradient of the stage input."""
        cfg, P = self.cfg, self.params
        dx = self.ws_dx
        if self.last:
            ops.gemm(self.logits, P.w("lm_head"), b_t=True, out=self.ws_dh)
            ops.gemm(self.logits, self.hf, a_t=True, b_t=True, out=P.g("lm_head"), accumulate=True)
            ops.rmsnorm_bwd(self.xs[-1], P.w("final_norm"), self.rstd_f, self.ws_dh, P.g("final_norm"), out=dx)
        else:
            dx.copy_(dx_top)
        for i in reversed(range(len(self.layer_ids))):
            l = self.layer_ids[i]
            p = f"layers.{l}."
            # MLP
            if self.f8 is not None:  # wgrad input: the activation recomputed and quantised in one pass
                from ..ops import fp8

                dyq = self.f8.quant_dy(l, "fc2", dx)
                fp8.gemm(dyq.rowwise(), self.f8.weight(l, "fc2").colwise(), out=self.ws_da)
                aq = self.f8.act_quant_cols(self.gu[i], cfg.gated)
                fp8.gemm(dyq.colwise(), aq.colwise(), out=P.g(p + "w2"), accumulate=True)
            else:
                mlp_act_fwd(cfg, self.gu[i], self.ws_a)
                self._linear_bwd(l, "fc2", dx, self.ws_a, P.w(p + "w2"), self.ws_da, P.g(p + "w2"))
            mlp_act_bwd(cfg, self.gu[i], self.ws_da, self.gu[i])
            dgu = self.gu[i]
            h2, _ = self._rmsnorm(self.x2[i], P.w(p + "mlp_norm"), self.ws_h, self.rstd2[i])
            self._linear_bwd(l, "fc1", dgu, h2, P.w(p + self.fc1), self.ws_dh, P.g(p + self.fc1))
            ops.rmsnorm_bwd(self.x2[i], P.w(p + "mlp_norm"), self.rstd2[i], self.ws_dh, P.g(p + "mlp_norm"), dres=dx,
                            out=self.ws_dx2)
            dx2 = self.ws_dx2
            # attention
            self._linear_bwd(l, "o", dx2, self.o[i], P.w(p + "wo"), self.ws_do, P.g(p + "wo"))
            q, k, v = self._views(i)
            D = cfg.head_dim
            dq = self.ws_dqkv[:, : cfg.heads * D]
            dk = self.ws_dqkv[:, cfg.heads * D: (cfg.heads + cfg.kv_heads) * D]
            dv = self.ws_dqkv[:, (cfg.heads + cfg.kv_heads) * D:]
            ops.attention_bwd(q, k, v, self.o[i], self.ws_do, self.lse[i], dq, dk, dv, **self._attn_kw())
            ops.rope_(dq, cfg.heads, D, self.cos, self.sin, self.S, inverse=True)
            ops.rope_(dk, cfg.kv_heads, D, self.cos, self.sin, self.S, inverse=True)
            h, _ = self._rmsnorm(self.xs[i], P.w(p + "attn_norm"), self.ws_h, self.rstd1[i])
            self._linear_bwd(l, "qkv", self.ws_dqkv, h, P.w(p + "wqkv"), self.ws_dh, P.g(p + "wqkv"))
            ops.rmsnorm_bwd(self.xs[i], P.w(p + "attn_norm"), self.rstd1[i], self.ws_dh, P.g(p + "attn_norm"),
                            dres=dx2, out=dx)
        if self.first:
            ops.embedding_bwd(ids, dx, P.g("embed"))
        return dx

    # ------------------------------------------------------------------ training step pieces
    def forward_backward(self, ids: torch.Tensor, labels: torch.Tensor, grad_scale: float) -> torch.Tensor:
        """One micro-batch on a single device holding every layer; accumulates gradients and
        adds the summed token loss into ``self.loss_acc``."""
        self.forward(ids)
        loss = self.head_loss(labels, grad_scale)
        self.loss_acc += loss.sum()
        self.backward(ids)
        return self.loss_acc

    def optimizer_step(self, lr: float, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0,
                       grad_scale: float = 1.0) -> None:
        P = self.params
        P.step += 1
        ops.adam_step(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.bf16, lr=lr, beta1=betas[0], beta2=betas[1],
                      eps=eps, weight_decay=weight_decay, step=P.step, grad_scale=grad_scale, zero_grad=True)
