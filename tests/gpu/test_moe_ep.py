"""Expert-parallel MoE layer with emulated ranks on one GPU (each phase's kernels run rank by rank;
none waits on another launch): forward and backward against fp32 autograd of the same layer
over all ranks' tokens."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _reference(xs, router_w, w13s, w2s, k, douts):
    x = torch.cat(xs).float().requires_grad_(True)
    rw = router_w.float().requires_grad_(True)
    w13 = [w.float().requires_grad_(True) for w in w13s]
    w2 = [w.float().requires_grad_(True) for w in w2s]
    logits = x @ rw.t()
    topi = logits.topk(k, dim=-1).indices
    gates = torch.softmax(logits.gather(-1, topi), dim=-1)
    out = x.clone()
    for e in range(len(w13)):
        rows, slot = (topi == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        gu = x[rows] @ w13[e].t()
        f = gu.shape[1] // 2
        a = F.silu(gu[:, :f]) * gu[:, f:]
        out = out.index_add(0, rows, gates[rows, slot].unsqueeze(1) * (a @ w2[e].t()))
    out.backward(torch.cat(douts).float())
    return out.detach(), x.grad, rw.grad, [w.grad for w in w13], [w.grad for w in w2], topi


@pytest.mark.parametrize("world,E,k,holder,speeds", [
    (4, 8, 2, None, None), (2, 4, 2, None, None), (8, 8, 2, None, None),
    # replicated experts: the pairs of experts 0 and 3 are dealt to two ranks by speed
    (4, 4, 2, [[0, 1], [1], [2], [3, 0]], {1: 0.5}),
])
def test_expert_parallel_layer_forward_backward(world, E, k, holder, speeds):
    from resihp_megatron_b200.ops.gemm import error_state
    from resihp_megatron_b200.parallel.moe_ep import ExpertParallelMoE

    H, Fd, T = 256, 512, 96
    torch.manual_seed(0)
    holder = holder or [e * world // E for e in range(E)]
    ranks = ExpertParallelMoE.emulated_group(world, "cuda", hidden=H, num_experts=E, top_k=k, max_tokens=T,
                                             holder=holder, speeds=speeds)
    xs = [torch.randn(T, H, device="cuda").bfloat16() for _ in range(world)]
    router_w = (torch.randn(E, H, device="cuda") / H ** 0.5).bfloat16()
    w13s = [(torch.randn(2 * Fd, H, device="cuda") / H ** 0.5).bfloat16() for _ in range(E)]
    w2s = [(torch.randn(H, Fd, device="cuda") / Fd ** 0.5).bfloat16() for _ in range(E)]
    douts = [torch.randn(T, H, device="cuda").bfloat16() for _ in range(world)]
    weights = {e: (w13s[e], w2s[e]) for e in range(E)}
    for r, m in enumerate(ranks):
        m.route(xs[r], router_w)
    table = torch.stack([m.heap.tensor("counts")[r * 16:r * 16 + E] for r, m in enumerate(ranks)])
    for m in ranks:
        m.set_counts_table(table)
    for m in ranks:
        m.dispatch()
    for m in ranks:
        m.experts_forward(weights)
    outs = [m.combine(xs[r]) for r, m in enumerate(ranks)]
    grads = {e: (torch.zeros(2 * Fd, H, device="cuda"), torch.zeros(H, Fd, device="cuda")) for e in range(E)}
    for r, m in enumerate(ranks):
        m.grad_push(douts[r])
    for m in ranks:
        m.experts_backward(weights, grads)
    rgrad = torch.zeros(E, H, device="cuda")
    dxs = [m.grad_pull(router_w, rgrad) for m in ranks]
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    out_ref, dx_ref, drw_ref, dw13_ref, dw2_ref, topi = _reference(xs, router_w, w13s, w2s, k, douts)
    got_topi = torch.cat([m.saved["topi"].long() for m in ranks])
    assert torch.equal(got_topi.sort(-1).values, topi.sort(-1).values)

    def close(a, b, tol):
        return (a.float() - b).abs().max().item() <= tol * b.abs().max().item() + tol

    assert close(torch.cat(outs), out_ref, 2e-2)
    assert close(torch.cat(dxs), dx_ref, 3e-2)
    assert close(rgrad, drw_ref, 3e-2)
    for e in range(E):
        assert close(grads[e][0], dw13_ref[e], 3e-2), e
        assert close(grads[e][1], dw2_ref[e], 3e-2), e
    ranks[0].close()
