"""The tcgen05 attention forward against an fp32 reference and against the mma.sync kernel."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, B, S, Hq, Hkv, D):
    qh = q.float().view(B, S, Hq, D).transpose(1, 2)
    kh = k.float().view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    vh = v.float().view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    att = (qh @ kh.transpose(-1, -2)) / math.sqrt(D)
    att = att.masked_fill(torch.ones(S, S, device=q.device, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(att, -1)
    return (att.softmax(-1) @ vh).transpose(1, 2).reshape(B * S, Hq * D), lse


@pytest.mark.parametrize("B,S,Hq,Hkv,amp", [(2, 256, 4, 2, 1.0), (1, 1024, 4, 1, 1.0), (1, 512, 2, 2, 4.0)])
def test_tcgen05_attention_forward(B, S, Hq, Hkv, amp):
    from resihp_megatron_b200 import ops

    D = 128
    torch.manual_seed(0)
    qkv = (torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda") * amp).bfloat16()
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    kw = dict(batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    o, lse = ops.attention_fwd(q, k, v, impl=ops.ATTN_TCGEN05, **kw)
    o2, lse2 = ops.attention_fwd(q, k, v, impl=ops.ATTN_MMA, **kw)
    ref, ref_lse = _ref(q, k, v, B, S, Hq, Hkv, D)
    torch.cuda.synchronize()
    assert int(ops.error_state()[0]) == 0
    err = (o.float() - ref).abs().max().item()
    assert err < 2e-2 * ref.abs().max().item() + 1e-2, err
    assert (lse.view(B, Hq, S) - ref_lse).abs().max().item() < 1e-2
    assert (o.float() - o2.float()).abs().max().item() < 3e-2 * ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
def test_tcgen05_attention_forward_fma_exp2_shares(variant):
    """Every share of softmax exponentials on the FMA-pipe polynomial (0-3 of 8) against the fp32
    reference; the polynomial's relative error (8.6e-5) is below bf16 resolution, so the outputs
    stay within a bf16 rounding of the all-MUFU kernel."""
    from resihp_megatron_b200 import ops

    B, S, Hq, Hkv, D = 1, 768, 4, 2, 128
    torch.manual_seed(2)
    qkv = (torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda") * 2.0).bfloat16()
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:]
    kw = dict(batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    o, lse = ops.attention_fwd(q, k, v, impl=ops.ATTN_TCGEN05, variant=variant, **kw)
    o0, lse0 = ops.attention_fwd(q, k, v, impl=ops.ATTN_TCGEN05, variant=0, **kw)
    ref, ref_lse = _ref(q, k, v, B, S, Hq, Hkv, D)
    torch.cuda.synchronize()
    assert int(ops.error_state()[0]) == 0
    scale = ref.abs().max().item()
    assert (o.float() - ref).abs().max().item() < 2e-2 * scale + 1e-2
    assert (lse.view(B, Hq, S) - ref_lse).abs().max().item() < 1e-2
    assert (o.float() - o0.float()).abs().max().item() < 1e-2 * scale + 4e-3
    assert (lse - lse0).abs().max().item() < 1e-3


def _ref_grads(q, k, v, dout, B, S, Hq, Hkv, D):
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    o, _ = _ref(qf, kf, vf, B, S, Hq, Hkv, D)
    o.backward(dout.float())
    return qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("B,S,Hq,Hkv", [(1, 256, 2, 2), (2, 384, 4, 1), (1, 1024, 8, 2)])
def test_tcgen05_attention_backward(B, S, Hq, Hkv):
    """dQ/dK/dV of the tcgen05 kernels against fp32 autograd and the mma.sync kernels; two
    runs are bitwise equal (no atomics)."""
    from resihp_megatron_b200 import ops

    D = 128
    torch.manual_seed(1)
    q = torch.randn(B * S, Hq * D, device="cuda").bfloat16()
    k = torch.randn(B * S, Hkv * D, device="cuda").bfloat16()
    v = torch.randn(B * S, Hkv * D, device="cuda").bfloat16()
    dout = torch.randn(B * S, Hq * D, device="cuda").bfloat16()
    kw = dict(batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    o, lse = ops.attention_fwd(q, k, v, impl=ops.ATTN_MMA, **kw)
    outs = {}
    for name, impl in (("tc", ops.ATTN_TCGEN05), ("tc2", ops.ATTN_TCGEN05), ("mma", ops.ATTN_MMA)):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ops.attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, impl=impl, **kw)
        outs[name] = (dq, dk, dv)
    torch.cuda.synchronize()
    assert int(ops.error_state()[0]) == 0
    ref = _ref_grads(q, k, v, dout, B, S, Hq, Hkv, D)
    for got, want, mma, name in zip(outs["tc"], ref, outs["mma"], ("dq", "dk", "dv")):
        scale = want.abs().max().item()
        err = (got.float() - want).abs().max().item()
        assert err < 2e-2 * scale + 1e-2, (name, err, scale)
        assert (got.float() - mma.float()).abs().max().item() < 3e-2 * scale + 1e-2, name
    for a, b in zip(outs["tc"], outs["tc2"]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
def test_tcgen05_attention_backward_fma_exp2_shares(variant):
    """dQ/dK/dV with 0-3 of every 8 probability exponentials on the FMA-pipe polynomial against
    fp32 autograd and the all-MUFU kernels; each variant stays bitwise deterministic."""
    from resihp_megatron_b200 import ops

    B, S, Hq, Hkv, D = 1, 512, 4, 2, 128
    torch.manual_seed(3)
    q = torch.randn(B * S, Hq * D, device="cuda").bfloat16()
    k = torch.randn(B * S, Hkv * D, device="cuda").bfloat16()
    v = torch.randn(B * S, Hkv * D, device="cuda").bfloat16()
    dout = torch.randn(B * S, Hq * D, device="cuda").bfloat16()
    kw = dict(batch=B, seq=S, heads=Hq, kv_heads=Hkv, head_dim=D)
    o, lse = ops.attention_fwd(q, k, v, impl=ops.ATTN_TCGEN05, variant=0, **kw)
    outs = []
    for var in (variant, variant, 0):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ops.attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, impl=ops.ATTN_TCGEN05, variant=var, **kw)
        outs.append((dq, dk, dv))
    torch.cuda.synchronize()
    assert int(ops.error_state()[0]) == 0
    ref = _ref_grads(q, k, v, dout, B, S, Hq, Hkv, D)
    for got, again, mufu, want, name in zip(outs[0], outs[1], outs[2], ref, ("dq", "dk", "dv")):
        scale = want.abs().max().item()
        assert (got.float() - want).abs().max().item() < 2e-2 * scale + 1e-2, name
        assert (got.float() - mufu.float()).abs().max().item() < 1e-2 * scale + 4e-3, name
        assert torch.equal(got, again), name
