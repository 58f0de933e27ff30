"""Fused tensor-parallel collective sweep (benchmark config 5, second half): all-gather -> GEMM and
GEMM -> reduce-scatter for M = 8192 tokens, K = N = 8192, at tp = 2, 4, 8 GPUs of one node.

* all-gather -> GEMM (column-parallel, sequence-parallel input): each rank holds ``[M / tp, K]``
  tokens and ``[N / tp, K]`` weight rows; result ``[M, N / tp]``.
  ``fused``: ``parallel.tp_fused.all_gather_gemm``; ``nccl``: ``all_gather_into_tensor`` then the
  same tcgen05 GEMM.
* GEMM -> reduce-scatter (row-parallel): each rank holds ``[M, K / tp]`` and ``[N, K / tp]``;
  result ``[M / tp, N]``.  ``fused``: ``gemm_reduce_scatter``; ``nccl``: the GEMM to a full
  ``[M, N]`` bf16 output then ``reduce_scatter_tensor``.

Device time per call is the median over iterations of the max over ranks (CUDA events with a
barrier + synchronize around each).  Roofline: the slower of FLOPs / measured cuBLAS bf16 peak and
the bytes that cross NVLink into (all-gather) or out of (reduce-scatter) one GPU at 770 GB/s.
Ranks outside a tp group idle for that row.  One JSON line per (op, tp, impl) from rank 0.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m resihp_megatron_b200.bench.tp_sweep
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _peak_tflops() -> float:
    from .kernels import peaks

    return peaks()["bf16_tflops"]


def _time(fn, iters: int, group) -> float:
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        dist.barrier(group=group)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    t = torch.tensor([sorted(times)[len(times) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def run(M: int = 8192, K: int = 8192, N: int = 8192, tps=(2, 4, 8), iters: int = 10) -> list[dict]:
    from ..ops import gemm
    from ..parallel.symm import exchange_via_group
    from ..parallel.tp_fused import TensorParallelComm

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    peak = _peak_tflops()
    rows = []
    for tp in tps:
        if tp > world:
            continue
        groups = [dist.new_group(list(range(s, s + tp))) for s in range(0, world - world % tp, tp)]
        if rank >= len(groups) * tp:
            continue
        gi = rank // tp
        group, me = groups[gi], rank % tp
        comm = TensorParallelComm(me, tp, exchange_via_group(group), dev, max_rows=M, max_k=K, max_n=N)
        g = torch.Generator(device=dev).manual_seed(rank)
        # ---- all-gather -> GEMM
        x_loc = torch.randn(M // tp, K, device=dev, generator=g).bfloat16()
        w_col = torch.randn(N // tp, K, device=dev, generator=g).bfloat16()
        x_all = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
        y = torch.empty(M, N // tp, dtype=torch.bfloat16, device=dev)
        def ag_fused():
            comm.local_chunk(M, K).copy_(x_loc)  # the producer of x writes its rows into the gather buffer
            comm.all_gather_gemm(M, w_col, out=y)

        def ag_nccl():
            dist.all_gather_into_tensor(x_all, x_loc, group=group)
            gemm(x_all, w_col, out=y)

        ag_bytes = (tp - 1) / tp * M * K * 2
        ag_flops = 2.0 * M * (N // tp) * K
        # ---- GEMM -> reduce-scatter
        x_row = torch.randn(M, K // tp, device=dev, generator=g).bfloat16()
        w_row = torch.randn(N, K // tp, device=dev, generator=g).bfloat16()
        full = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        y_rs = torch.empty(M // tp, N, dtype=torch.bfloat16, device=dev)

        def rs_fused():
            comm.gemm_reduce_scatter(x_row, w_row, out=y_rs)

        def rs_nccl():
            gemm(x_row, w_row, out=full)
            dist.reduce_scatter_tensor(y_rs, full, group=group)

        rs_bytes = (tp - 1) / tp * M * N * 2
        rs_flops = 2.0 * M * N * (K // tp)
        # correctness of the fused paths against the NCCL ones
        ag_fused()
        ref = y.clone()
        ag_nccl()
        ag_ok = bool(torch.equal(ref, y))
        rs_fused()
        ref_rs = y_rs.float().clone()
        rs_nccl()
        rs_err = (ref_rs - y_rs.float()).abs().max().item() / (y_rs.float().abs().max().item() + 1e-6)
        comm.heap.check()  # a peer that missed a barrier ends the sweep here
        for op, fns, nbytes, flops in (("allgather_gemm", (("fused", ag_fused), ("nccl", ag_nccl)), ag_bytes, ag_flops),
                                       ("gemm_reducescatter", (("fused", rs_fused), ("nccl", rs_nccl)), rs_bytes,
                                        rs_flops)):
            for impl, fn in fns:
                ms = _time(fn, iters, group)
                roof = max(flops / (peak * 1e12), nbytes / (NVLINK_GBS * 1e9)) * 1e3
                row = {"op": op, "tp": tp, "impl": impl, "M": M, "K": K, "N": N, "ms": round(ms, 4),
                       "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / ms, 3),
                       "nvlink_MB_per_gpu": round(nbytes / 1e6, 1)}
                if impl == "fused":
                    row["matches_nccl_path"] = ag_ok if op == "allgather_gemm" else round(rs_err, 5)
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
        torch.cuda.synchronize()
        dist.barrier(group=group)
        comm.close()
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=8192)
    ap.add_argument("--K", type=int, default=8192)
    ap.add_argument("--N", type=int, default=8192)
    ap.add_argument("--tps", default="2,4,8")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    run(a.M, a.K, a.N, tuple(int(x) for x in a.tps.split(",")), a.iters)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
