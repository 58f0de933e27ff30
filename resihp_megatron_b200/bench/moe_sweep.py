"""Expert-parallel MoE layer on 8 GPUs (Mixtral-8x7B shapes, benchmark config 3's layer): hidden 4096,
8 SwiGLU experts of FFN 14336, top-2, one expert per GPU, 4096 tokens per GPU, uniform random
inputs.  Forward + backward of one layer:

* ``peer``: this framework's path (``parallel.moe_ep``): router kernel, fixed-order positions,
  dispatch / combine and their gradients as peer stores and loads over NVLink, counts pulled from
  the peers' memory, the same tcgen05 expert GEMMs;
* ``nccl``: the reference's transport (``resihp/runtime/moe.py:149-265``): a counts
  ``all_to_all_single``, token permutation, ``all_to_all_single`` dispatch and combine (and their
  transposes in the backward), ``index_add`` combine -- with the same router and expert kernels.

Device time (CUDA events, barrier + synchronize around each call), median over iterations, max
over ranks.  Rank 0 prints one JSON line per implementation.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m resihp_megatron_b200.bench.moe_sweep
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist


def run(H=4096, Fd=14336, E=8, k=2, T=4096, iters=5) -> list[dict]:
    from .. import ops
    from ..ops._build import ext
    from ..parallel.moe_ep import ExpertParallelMoE
    from ..parallel.symm import exchange_via_group

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    holder = [e * world // E for e in range(E)]
    local = [e for e in range(E) if holder[e] == rank]
    g = torch.Generator(device=dev).manual_seed(123)
    router_w = (torch.randn(E, H, device=dev, generator=g) / H ** 0.5).bfloat16()
    gl = torch.Generator(device=dev).manual_seed(1000 + rank)
    weights = {e: ((torch.randn(2 * Fd, H, device=dev, generator=gl) / H ** 0.5).bfloat16(),
                   (torch.randn(H, Fd, device=dev, generator=gl) / Fd ** 0.5).bfloat16()) for e in local}
    grads = {e: (torch.zeros(2 * Fd, H, device=dev), torch.zeros(H, Fd, device=dev)) for e in local}
    rgrad = torch.zeros(E, H, device=dev)
    x = torch.randn(T, H, device=dev, generator=gl).bfloat16()
    dout = torch.randn(T, H, device=dev, generator=gl).bfloat16()
    moe = ExpertParallelMoE(rank, world, exchange_via_group(), dev, hidden=H, num_experts=E, top_k=k, max_tokens=T,
                            holder=holder)

    def peer_step():
        moe.route(x, router_w)
        moe.exchange_counts()
        moe.dispatch()
        moe.experts_forward(weights)
        moe.combine(x)
        moe.finish_forward()
        moe.grad_push(dout)
        moe.experts_backward(weights, grads)
        moe.grad_pull(router_w, rgrad)

    def nccl_step():
        logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        topi = torch.empty(T, k, dtype=torch.int32, device=dev)
        gates = torch.empty(T, k, dtype=torch.float32, device=dev)
        ext().moe_route(x, router_w, None, k, logits, topi, gates)
        flat = topi.reshape(-1).long()
        dest = torch.tensor(holder, device=dev)[flat]
        order = torch.argsort(dest * E + flat, stable=True)
        send_counts = torch.bincount(dest, minlength=world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        tok = x[order // k]
        recv = torch.empty(sum(rc), H, dtype=torch.bfloat16, device=dev)
        dist.all_to_all_single(recv, tok, rc, sc)
        # experts: rows arrive grouped by source; one local expert per rank here
        e = local[0]
        w13, w2 = weights[e]
        gu = ops.gemm(recv, w13)
        a = ops.swiglu_fwd(gu)
        y = ops.gemm(a, w2)
        back = torch.empty_like(tok)
        dist.all_to_all_single(back, y, sc, rc)
        gsel = gates.reshape(-1)[order]
        out = x.clone().index_add_(0, order // k, (back.float() * gsel[:, None]).bfloat16())
        # backward transport: dy to experts, expert backward, dx back
        dy = (dout[order // k].float() * gsel[:, None]).bfloat16()
        dyr = torch.empty_like(recv)
        dist.all_to_all_single(dyr, dy, rc, sc)
        da = ops.gemm(dyr, w2, b_t=True)
        ops.gemm(dyr, a, a_t=True, b_t=True, out=grads[e][1], accumulate=True)
        dgu = ops.swiglu_bwd(gu, da)
        ops.gemm(dgu, recv, a_t=True, b_t=True, out=grads[e][0], accumulate=True)
        dxr = ops.gemm(dgu, w13, b_t=True)
        dxb = torch.empty_like(tok)
        dist.all_to_all_single(dxb, dxr, sc, rc)
        dx = dout.clone().index_add_(0, order // k, dxb)
        return out, dx

    rows = []
    for impl, fn in (("peer", peer_step), ("nccl", nccl_step)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        moe.heap.check()  # a peer that missed a barrier ends the sweep here
        times = []
        for _ in range(iters):
            dist.barrier()
            torch.cuda.synchronize()
            s, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e_.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e_))
        t = torch.tensor([sorted(times)[len(times) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        flops = 3 * 2.0 * T * k * 3 * H * Fd  # fwd + bwd expert GEMMs per GPU (balanced routing)
        row = {"op": "moe_layer_fwd_bwd", "impl": impl, "tokens_per_gpu": T, "hidden": H, "ffn": Fd, "experts": E,
               "top_k": k, "gpus": world, "ms": round(float(t.item()), 4),
               "expert_tflops_per_gpu": round(flops / float(t.item()) / 1e9, 1)}
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    moe.close()
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    run(T=a.tokens, iters=a.iters)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
