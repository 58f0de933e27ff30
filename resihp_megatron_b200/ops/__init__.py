"""Hand-written sm_100a kernels of the data plane and their Python entry points.

Every function here launches one of this package's own CUDA kernels (``ops/csrc``); none
falls back to a PyTorch implementation.  On a host without the extension the first call
raises.  Shapes follow the token-major convention of the model: activations are
``[T, features]`` with ``T = batch * seq``.
"""

from __future__ import annotations

import math

import torch

from ._build import ext
from .gemm import EPI_BF16, EPI_BF16_RES, EPI_F32, EPI_F32_ACC, error_state, gemm
from .counter import count, launches, reset_launches

__all__ = [
    "gemm", "error_state", "rmsnorm_fwd", "rmsnorm_bwd", "rope_", "swiglu_fwd", "swiglu_bwd", "embedding_fwd",
    "embedding_bwd", "gelu_fwd", "gelu_bwd", "adam_step", "sumsq", "cross_entropy_", "attention_fwd",
    "attention_bwd", "rope_tables", "EPI_BF16", "EPI_BF16_RES", "EPI_F32", "EPI_F32_ACC", "launches", "reset_launches",
]


def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5, out: torch.Tensor | None = None,
                rstd: torch.Tensor | None = None):
    """``y = x / rms(x) * w`` over the last dim; returns ``(y, rstd)`` (``rstd``: fp32 per row)."""
    H = x.shape[-1]
    y = torch.empty_like(x) if out is None else out
    if rstd is None:
        rstd = torch.empty(x.numel() // H, dtype=torch.float32, device=x.device)
    ext().rmsnorm_fwd(x, w, y, rstd, float(eps))
    count(1)
    return y, rstd


def rmsnorm_bwd(x, w, rstd, dy, dw: torch.Tensor, dres: torch.Tensor | None = None, accumulate: bool = True,
                out: torch.Tensor | None = None):
    """Input gradient (plus ``dres``, the residual-stream gradient, when given); ``dw`` (fp32)
    receives the weight gradient, added to its contents when ``accumulate``."""
    dx = torch.empty_like(x) if out is None else out
    ext().rmsnorm_bwd(x, w, rstd, dy, dres, dx, dw, bool(accumulate))
    count(2)
    return dx


def rope_tables(seq_len: int, head_dim: int, theta: float = 500000.0, device=None):
    """cos/sin tables ``[seq_len, head_dim // 2]`` (fp32) for rotate-half RoPE."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    pos = torch.arange(seq_len, dtype=torch.float64)
    ang = torch.outer(pos, inv)
    return ang.cos().float().to(device), ang.sin().float().to(device)


def rope_(t: torch.Tensor, heads: int, head_dim: int, cos_t, sin_t, seq_len: int, inverse: bool = False):
    """Rotate ``heads`` heads of a token-major 2-D view in place (``inverse`` undoes it)."""
    assert t.dim() == 2 and t.stride(1) == 1
    ext().rope(t, t.stride(0), heads, head_dim, cos_t, sin_t, seq_len, t.shape[0], bool(inverse))
    count(1)
    return t


def swiglu_fwd(gu: torch.Tensor, out: torch.Tensor | None = None):
    """``gu = [T, 2F]`` (gate | up) -> ``silu(gate) * up`` of shape ``[T, F]``."""
    T, F2 = gu.shape
    a = torch.empty((T, F2 // 2), dtype=gu.dtype, device=gu.device) if out is None else out
    ext().swiglu_fwd(gu, a)
    count(1)
    return a


def swiglu_bwd(gu: torch.Tensor, da: torch.Tensor, out: torch.Tensor | None = None):
    """Gradient w.r.t. ``gu``; ``out`` may alias ``gu`` (in place)."""
    dgu = torch.empty_like(gu) if out is None else out
    ext().swiglu_bwd(gu, da, dgu)
    count(1)
    return dgu


def gelu_fwd(h: torch.Tensor, out: torch.Tensor | None = None):
    """GELU (tanh form) of a bf16 tensor."""
    a = torch.empty_like(h) if out is None else out
    ext().gelu_fwd(h, a)
    count(1)
    return a


def gelu_bwd(h: torch.Tensor, da: torch.Tensor, out: torch.Tensor | None = None):
    """``da * gelu'(h)``; ``out`` may alias ``h`` (in place)."""
    dh = torch.empty_like(h) if out is None else out
    ext().gelu_bwd(h, da, dh)
    count(1)
    return dh


def embedding_fwd(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None):
    ids = ids.reshape(-1).contiguous()
    x = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device) if out is None else out
    ext().embedding_fwd(ids, table, x)
    count(1)
    return x


def embedding_bwd(ids: torch.Tensor, dx: torch.Tensor, dtable: torch.Tensor):
    """``dtable[ids[t]] += dx[t]`` in a fixed (id, position) order -- deterministic."""
    ext().embedding_bwd(ids.reshape(-1).contiguous(), dx, dtable)
    count(1)
    return dtable


def adam_step(p, grad, m, v, p_bf16=None, *, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0,
              decoupled=False, step: int, grad_scale=1.0, zero_grad=False, bias_corr: torch.Tensor | None = None):
    """Fused Adam(W) on flat fp32 buffers; optionally refreshes a bf16 copy of the weights.
    ``bias_corr`` (fp32 device ``[1 - beta1^t, sqrt(1 - beta2^t)]``) is read by the kernel
    instead of ``step``'s host values -- for CUDA graphs, whose replays keep launch arguments."""
    ext().adam_step(p, grad, m, v, p_bf16, float(lr), float(beta1), float(beta2), float(eps), float(weight_decay),
                    bool(decoupled), int(step), float(grad_scale), bool(zero_grad), bias_corr)
    count(1)


def sumsq(x: torch.Tensor) -> torch.Tensor:
    """Deterministic sum of squares of a flat fp32 buffer (0-d fp32 tensor)."""
    count(1)
    return ext().sumsq(x)


def cross_entropy_(logits: torch.Tensor, labels: torch.Tensor, *, grad_scale: float = 1.0, ignore_index: int = -100,
                   write_grad: bool = True, vocab_start: int = 0, lse: torch.Tensor | None = None):
    """Per-token loss (fp32 ``[T]``); the logits are overwritten by ``dloss/dlogits * grad_scale``."""
    loss = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
    ext().cross_entropy(logits, labels.reshape(-1).contiguous(), loss, lse, int(vocab_start), float(grad_scale),
                        int(ignore_index), bool(write_grad))
    count(1)
    return loss


ATTN_AUTO, ATTN_MMA, ATTN_TCGEN05 = 0, 1, 2


def attention_fwd(q, k, v, *, batch: int, seq: int, heads: int, kv_heads: int, head_dim: int, causal: bool = True,
                  scale: float | None = None, out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                  impl: int = ATTN_AUTO, variant: int = -1):
    """Causal GQA attention on token-major 2-D views; returns ``(o, lse)``.  ``impl``: the
    tcgen05 kernel (head dim 128, causal, seq % 256 == 0) with the mma.sync kernel for other
    shapes (``ATTN_AUTO``), or one of them explicitly.  ``variant`` (tcgen05 kernel, tuning):
    how many of every 8 softmax exponentials run as an FMA-pipe polynomial instead of on the
    MUFU unit (0-3; -1 = the built-in default)."""
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    o = torch.empty((q.shape[0], heads * head_dim), dtype=q.dtype, device=q.device) if out is None else out
    if lse is None:
        lse = torch.empty((batch, heads, seq), dtype=torch.float32, device=q.device)
    ext().attention_fwd(q, k, v, o, lse, batch, seq, heads, kv_heads, head_dim, float(scale), bool(causal), int(impl),
                        int(variant))
    count(1)
    return o, lse


def attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, *, batch: int, seq: int, heads: int, kv_heads: int,
                  head_dim: int, causal: bool = True, scale: float | None = None, impl: int = ATTN_AUTO,
                  variant: int = -1):
    """Writes dq/dk/dv (token-major 2-D views, may be column slices of one buffer).  ``impl`` as
    in ``attention_fwd``: the tcgen05 kernels (head dim 128, causal, seq % 128 == 0) or the
    mma.sync kernels."""
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    delta = torch.empty((batch, heads, seq), dtype=torch.float32, device=q.device)
    ext().attention_bwd(q, k, v, o, dout, lse, delta, dq, dk, dv, batch, seq, heads, kv_heads, head_dim, float(scale),
                        bool(causal), int(impl), int(variant))
    count(3)
