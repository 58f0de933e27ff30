"""Numerics of the bandwidth-bound kernels and attention against fp32 PyTorch references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def test_rmsnorm_fwd_bwd():
    from resihp_megatron_b200 import ops

    T, H = 300, 4096
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    dy = torch.randn(T, H, device="cuda").bfloat16()
    dres = torch.randn(T, H, device="cuda").bfloat16()
    y, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * wf
    assert rel(y, ref) < 1e-2
    ref.backward(dy.float())
    dw = torch.zeros(H, device="cuda")
    dx = ops.rmsnorm_bwd(x, w, rstd, dy, dw, dres=dres)
    assert rel(dx, xf.grad + dres.float()) < 1e-2
    assert rel(dw, wf.grad) < 1e-3
    dw2 = torch.full((H,), 1.0, device="cuda")
    ops.rmsnorm_bwd(x, w, rstd, dy, dw2, accumulate=True)
    assert rel(dw2 - 1.0, wf.grad) < 1e-3


def test_rope_roundtrip_and_reference():
    from resihp_megatron_b200 import ops

    S, B, Hh, D = 64, 2, 4, 128
    cos, sin = ops.rope_tables(S, D, device="cuda")
    x = torch.randn(B * S, Hh * D, device="cuda").bfloat16()
    y = x.clone()
    ops.rope_(y, Hh, D, cos, sin, S)
    xf = x.float().view(B, S, Hh, D)
    c = cos.view(1, S, 1, D // 2).repeat(1, 1, 1, 2)
    s = sin.view(1, S, 1, D // 2).repeat(1, 1, 1, 2)
    rot = torch.cat([-xf[..., D // 2:], xf[..., : D // 2]], -1)
    ref = (xf * c + rot * s).view(B * S, Hh * D)
    assert rel(y, ref) < 1e-2
    ops.rope_(y, Hh, D, cos, sin, S, inverse=True)
    assert rel(y, x) < 2e-2


def test_swiglu():
    from resihp_megatron_b200 import ops

    T, F = 100, 1024
    gu = torch.randn(T, 2 * F, device="cuda").bfloat16()
    da = torch.randn(T, F, device="cuda").bfloat16()
    a = ops.swiglu_fwd(gu)
    g = gu.float().requires_grad_(True)
    ref = torch.nn.functional.silu(g[:, :F]) * g[:, F:]
    assert rel(a, ref) < 1e-2
    ref.backward(da.float())
    dgu = ops.swiglu_bwd(gu, da)
    assert rel(dgu, g.grad) < 1e-2


def test_embedding_deterministic():
    from resihp_megatron_b200 import ops

    V, H, T = 1000, 256, 777
    E = torch.randn(V, H, device="cuda").bfloat16()
    ids = torch.randint(0, 50, (T,), device="cuda")
    x = ops.embedding_fwd(ids, E)
    assert torch.equal(x, E[ids])
    dx = torch.randn(T, H, device="cuda").bfloat16()
    d1 = torch.zeros(V, H, device="cuda")
    d2 = torch.zeros(V, H, device="cuda")
    ops.embedding_bwd(ids, dx, d1)
    ops.embedding_bwd(ids, dx, d2)
    ref = torch.zeros(V, H, device="cuda").index_add_(0, ids, dx.float())
    assert torch.equal(d1, d2)
    assert rel(d1, ref) < 1e-5


def test_adam_matches_torch():
    from resihp_megatron_b200 import ops

    n = 10003
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    tp = p.clone().requires_grad_(True)
    opt = torch.optim.Adam([tp], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, foreach=False)
    for step in range(1, 4):
        tp.grad = g.clone() * 0.5
        opt.step()
        ops.adam_step(p, g, m, v, pb, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, step=step, grad_scale=0.5)
    assert rel(p, tp.detach()) < 1e-6
    assert torch.equal(pb, p.bfloat16())


def test_cross_entropy():
    from resihp_megatron_b200 import ops

    T, V = 37, 50257
    logits = torch.randn(T, V, device="cuda").bfloat16()
    labels = torch.randint(0, V, (T,), device="cuda")
    labels[3] = -100
    lf = logits.float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(lf, labels, reduction="none", ignore_index=-100)
    ref.sum().backward()
    work = logits.clone()
    loss = ops.cross_entropy_(work, labels, grad_scale=1.0)
    assert rel(loss, ref) < 1e-3
    assert (work.float() - lf.grad).abs().max().item() < 2e-2 * lf.grad.abs().max().item() + 1e-3


@pytest.mark.parametrize("S,Hq,Hkv,D", [(256, 4, 2, 128), (200, 4, 4, 64), (130, 8, 2, 128)])
def test_attention_fwd_bwd(S, Hq, Hkv, D):
    from resihp_megatron_b200 import ops

    B = 2
    torch.manual_seed(0)
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    q = qkv[:, : Hq * D]
    k = qkv[:, Hq * D: (Hq + Hkv) * D]
    v = qkv[:, (Hq + Hkv) * D:]
    o, lse = ops.attention_fwd(q, k, v, batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)

    def ref_attn(qf, kf, vf):
        qh = qf.view(B, S, Hq, D).transpose(1, 2)
        kh = kf.view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
        vh = vf.view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
        att = (qh @ kh.transpose(-1, -2)) / math.sqrt(D)
        mask = torch.ones(S, S, device="cuda", dtype=torch.bool).triu(1)
        att = att.masked_fill(mask, float("-inf")).softmax(-1)
        return (att @ vh).transpose(1, 2).reshape(B * S, Hq * D)

    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    ref = ref_attn(qf, kf, vf)
    assert rel(o, ref) < 2e-2
    do = torch.randn_like(o)
    ref.backward(do.float())
    dqkv = torch.empty_like(qkv)
    dq, dk, dv = dqkv[:, : Hq * D], dqkv[:, Hq * D: (Hq + Hkv) * D], dqkv[:, (Hq + Hkv) * D:]
    ops.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    assert rel(dq, qf.grad) < 3e-2
    assert rel(dk, kf.grad) < 3e-2
    assert rel(dv, vf.grad) < 3e-2
    # deterministic
    dqkv2 = torch.empty_like(qkv)
    ops.attention_bwd(q, k, v, o, do, lse, dqkv2[:, : Hq * D], dqkv2[:, Hq * D: (Hq + Hkv) * D],
                      dqkv2[:, (Hq + Hkv) * D:], batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    assert torch.equal(dqkv, dqkv2)


def test_adam_bias_corrections_from_device_equal_the_host_step():
    import math

    from resihp_megatron_b200 import ops

    n, step, b1, b2 = 4099, 7, 0.9, 0.95
    torch.manual_seed(1)
    p0, g = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
    m0, v0 = torch.randn(n, device="cuda") * 0.1, torch.rand(n, device="cuda") * 0.1
    outs = []
    for dev in (False, True):
        p, m, v = p0.clone(), m0.clone(), v0.clone()
        bc = torch.tensor([1 - b1 ** step, math.sqrt(1 - b2 ** step)], dtype=torch.float32, device="cuda")
        ops.adam_step(p, g, m, v, lr=1e-3, beta1=b1, beta2=b2, step=1 if dev else step, bias_corr=bc if dev else None)
        outs.append((p, m, v))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
