"""PyTorch stand-ins for the data-plane kernels, for CPU tests of the orchestration around them.

Same signatures and in-place semantics as ``resihp_megatron_b200.ops`` (fp32 math, results
rounded to the output dtype).  ``install(monkeypatch)`` swaps them into the ``ops`` module so
that GPU-stage code (``models.tp_stage``, ``runtime.gpu_runtime``) runs on gloo ranks; the
kernels themselves are tested against fp32 references in ``tests/gpu``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def gemm(a, b, *, a_t=False, b_t=False, out=None, out_dtype=torch.bfloat16, accumulate=False, residual=None,
         alpha=1.0, variant=0):
    A = (a.t() if a_t else a).float()
    Bop = (b.t() if b_t else b).float()  # op(b) is [N, K]
    r = alpha * (A @ Bop.t())
    if accumulate:
        out += r
        return out
    if residual is not None:
        r = r + residual.float()
    if out is None:
        out = torch.empty(r.shape, dtype=torch.float32 if out_dtype == torch.float32 else torch.bfloat16)
    out.copy_(r)
    return out


def rmsnorm_fwd(x, w, eps=1e-5, out=None, rstd=None):
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    y = xf * r[:, None] * w.float()
    out = torch.empty_like(x) if out is None else out
    rstd = torch.empty(x.shape[0], dtype=torch.float32) if rstd is None else rstd
    out.copy_(y)
    rstd.copy_(r)
    return out, rstd


def rmsnorm_bwd(x, w, rstd, dy, dw, dres=None, accumulate=True, out=None):
    xf, dyf, r = x.float(), dy.float(), rstd.float()
    xhat = xf * r[:, None]
    part = (dyf * xhat).sum(0)
    if accumulate:
        dw += part
    else:
        dw.copy_(part)
    g = dyf * w.float()
    dx = r[:, None] * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    if dres is not None:
        dx = dx + dres.float()
    out = torch.empty_like(x) if out is None else out
    out.copy_(dx)
    return out


def rope_tables(seq_len, head_dim, theta=500000.0, device=None):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.outer(torch.arange(seq_len, dtype=torch.float64), inv)
    return ang.cos().float(), ang.sin().float()


def rope_(t, heads, head_dim, cos_t, sin_t, seq_len, inverse=False):
    T, h = t.shape[0], head_dim // 2
    v = t.unflatten(1, (heads, head_dim))
    pos = torch.arange(T) % seq_len
    c, s = cos_t[pos][:, None, :], sin_t[pos][:, None, :]
    if inverse:
        s = -s
    x1, x2 = v[..., :h].float(), v[..., h:].float()
    o1, o2 = x1 * c - x2 * s, x2 * c + x1 * s
    v[..., :h] = o1.to(t.dtype)
    v[..., h:] = o2.to(t.dtype)
    return t


def swiglu_fwd(gu, out=None):
    Fh = gu.shape[1] // 2
    a = F.silu(gu[:, :Fh].float()) * gu[:, Fh:].float()
    out = torch.empty(gu.shape[0], Fh, dtype=gu.dtype) if out is None else out
    out.copy_(a)
    return out


def swiglu_bwd(gu, da, out=None):
    Fh = gu.shape[1] // 2
    g, u, d = gu[:, :Fh].float(), gu[:, Fh:].float(), da.float()
    sig = torch.sigmoid(g)
    dg = d * u * sig * (1 + g * (1 - sig))
    du = d * g * sig
    res = torch.cat([dg, du], 1)
    out = torch.empty_like(gu) if out is None else out
    out.copy_(res)
    return out


def embedding_fwd(ids, table, out=None):
    r = table[ids.reshape(-1)]
    if out is None:
        return r.clone()
    out.copy_(r)
    return out


def embedding_bwd(ids, dx, dtable):
    dtable.index_add_(0, ids.reshape(-1), dx.float())
    return dtable


def cross_entropy_(logits, labels, *, grad_scale=1.0, ignore_index=-100, write_grad=True, vocab_start=0, lse=None):
    lf = logits.float()
    lab = labels.reshape(-1)
    lz = torch.logsumexp(lf, -1)
    loss = lz - lf.gather(1, lab[:, None]).squeeze(1)
    if write_grad:
        p = torch.softmax(lf, -1)
        p[torch.arange(p.shape[0]), lab] -= 1.0
        logits.copy_(p * grad_scale)
    return loss


def _attn(q, k, v, batch, seq, heads, kv_heads, head_dim, causal, scale):
    qf = q.reshape(batch, seq, heads, head_dim).transpose(1, 2)
    kf = k.reshape(batch, seq, kv_heads, head_dim).transpose(1, 2).repeat_interleave(heads // kv_heads, 1)
    vf = v.reshape(batch, seq, kv_heads, head_dim).transpose(1, 2).repeat_interleave(heads // kv_heads, 1)
    att = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        att = att.masked_fill(torch.ones(seq, seq, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(att, -1)
    o = (att.softmax(-1) @ vf).transpose(1, 2).reshape(batch * seq, heads * head_dim)
    return o, lse


def attention_fwd(q, k, v, *, batch, seq, heads, kv_heads, head_dim, causal=True, scale=None, out=None, lse=None,
                  impl=0):
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    o, l = _attn(q.float(), k.float(), v.float(), batch, seq, heads, kv_heads, head_dim, causal, scale)
    out = torch.empty(q.shape[0], heads * head_dim, dtype=q.dtype) if out is None else out
    lse = torch.empty(batch, heads, seq) if lse is None else lse
    out.copy_(o)
    lse.copy_(l)
    return out, lse


def attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, *, batch, seq, heads, kv_heads, head_dim, causal=True,
                  scale=None, impl=0):
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    qf, kf, vf = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    of, _ = _attn(qf, kf, vf, batch, seq, heads, kv_heads, head_dim, causal, scale)
    of.backward(dout.float())
    dq.copy_(qf.grad)
    dk.copy_(kf.grad)
    dv.copy_(vf.grad)


def adam_step(p, grad, m, v, p_bf16=None, *, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0,
              decoupled=False, step, grad_scale=1.0, zero_grad=False, bias_corr=None):
    bc1, bc2s = 1 - beta1 ** step, math.sqrt(1 - beta2 ** step)
    if bias_corr is not None:
        bc1, bc2s = float(bias_corr[0]), float(bias_corr[1])
    g = grad * grad_scale
    if weight_decay:
        if decoupled:
            p.mul_(1 - lr * weight_decay)
        else:
            g = g + weight_decay * p
    m.add_((1 - beta1) * (g - m))
    v.mul_(beta2).add_((1 - beta2) * g * g)
    p.sub_((lr / bc1) * (m / (v.sqrt() / bc2s + eps)))
    if zero_grad:
        grad.zero_()
    if p_bf16 is not None:
        p_bf16.copy_(p)


def gelu_fwd(h, out=None):
    a = F.gelu(h.float(), approximate="tanh")
    out = torch.empty_like(h) if out is None else out
    out.copy_(a)
    return out


def gelu_bwd(h, da, out=None):
    x = h.float().clone().requires_grad_(True)
    F.gelu(x, approximate="tanh").backward(da.float())
    out = torch.empty_like(h) if out is None else out
    out.copy_(x.grad)
    return out


# block-scaled fp8: the PyTorch emulation of the kernels (bit-exact quantiser)
def fp8_quantize(x, fmt=0, *, two_d=False, rowwise=True, colwise=False, amax=None, out=None, row_major=False,
                 act=None):
    from resihp_megatron_b200.ops import fp8

    if act is not None:
        x = swiglu_fwd(x) if act == "swiglu" else gelu_fwd(x)
    if out is not None:
        row_major = out.row_major
    ref = fp8.quantize_reference(x, fmt, two_d=two_d, rowwise=rowwise, colwise=colwise, amax=amax,
                                 row_major=row_major)
    if out is None:
        return ref
    for name in ("q_row", "s_row", "q_col", "s_col"):
        src, dst = getattr(ref, name), getattr(out, name)
        if src is not None and dst is not None:
            dst.copy_(src)
    return out


def fp8_rmsnorm_quantize(x, w, eps, fmt=0, *, out, rstd=None, amax=None):
    y, r = rmsnorm_fwd(x, w, eps, rstd=rstd)
    return fp8_quantize(y, fmt, rowwise=True, amax=amax, out=out)


def fp8_act_quantize(x, gated, fmt=0, *, out, amax=None):
    y = swiglu_fwd(x) if gated else gelu_fwd(x)
    return fp8_quantize(y, fmt, rowwise=True, amax=amax, out=out)


def fp8_gemm(a, b, *, out=None, out_dtype=torch.bfloat16, accumulate=False, alpha=1.0, residual=None, scatter=None):
    from resihp_megatron_b200.ops import fp8

    if scatter is not None:
        raise NotImplementedError("the scatter epilogue writes peer memory (GPU only)")
    return fp8.gemm_reference(a, b, out=out, out_dtype=out_dtype, accumulate=accumulate, alpha=alpha,
                              residual=residual)


def fp8_amax_history_push(history, pending):
    from resihp_megatron_b200.ops import fp8

    fp8.amax_history_push_reference(history, pending)


NAMES = ("gemm", "rmsnorm_fwd", "rmsnorm_bwd", "rope_tables", "rope_", "swiglu_fwd", "swiglu_bwd", "embedding_fwd",
         "embedding_bwd", "cross_entropy_", "attention_fwd", "attention_bwd", "adam_step", "gelu_fwd", "gelu_bwd")
FP8_NAMES = {"quantize": fp8_quantize, "gemm": fp8_gemm, "amax_history_push": fp8_amax_history_push,
             "rmsnorm_quantize": fp8_rmsnorm_quantize, "act_quantize": fp8_act_quantize}


def install(monkeypatch=None) -> None:
    """Swap the stand-ins into ``resihp_megatron_b200.ops`` and ``ops.fp8`` (with ``monkeypatch``
    when given, so a test undoes it; plain assignment in a spawned worker process)."""
    from resihp_megatron_b200 import ops
    from resihp_megatron_b200.ops import fp8

    g = globals()
    targets = [(ops, n, g[n]) for n in NAMES] + [(fp8, n, f) for n, f in FP8_NAMES.items()]
    for mod, n, f in targets:
        if monkeypatch is not None:
            monkeypatch.setattr(mod, n, f)
        else:
            setattr(mod, n, f)
