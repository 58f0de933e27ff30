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
