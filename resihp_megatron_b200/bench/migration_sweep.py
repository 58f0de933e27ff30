"""Live-migration sweep (benchmark config 5, first half): reshard a bf16 ``[N, N]`` weight plus two
fp32 Adam moments from TP8 -> TP4 -> TP2 (row shards, the column-parallel layout), N in {4096,
8192, 16384}, values N(0, 1) from seed 0, on 8 GPUs of one node.

Two implementations of the same transfer plan (``state.transfer_plan.plan_transfers`` over the
old and new holdings, so the pieces, sources and destinations are those of a real
reconfiguration):

* ``peer``  -- this framework: the old shards live in the symmetric heap; every new owner pulls
  all of its pieces (weight and both moments) from the old owners' memory with ONE slice-copy
  kernel (``ops/csrc/symm.cu``), then a bounded barrier;
* ``nccl``  -- the reference's path (``resihp/state/transfer_engine.py:24-59``): one
  isend/irecv per (piece, kind) over NCCL, local pieces copied.

Device time per transition is the max over ranks (CUDA events, barrier + synchronize on both
sides).  Roofline: bytes that must cross NVLink into the busiest rank / 770 GB/s (the measured
per-direction peer copy rate on this pool).  Rank 0 prints one JSON line per (N, transition, impl).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m resihp_megatron_b200.bench.migration_sweep
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def shards(n: int, parts: int) -> list[tuple[int, int]]:
    from ..utils.intervals import even_split

    return even_split(n, parts)


def run(sizes=(4096, 8192, 16384), iters: int = 5) -> list[dict]:
    from ..ops._build import ext
    from ..parallel.symm import SymmetricHeap, exchange_via_group
    from ..state.transfer_plan import plan_transfers

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    ids = [f"g{r}" for r in range(world)]
    rows = []
    for N in sizes:
        for old_tp, new_tp in ((8, 4), (4, 2)):
            if old_tp > world:
                continue
            old_iv = shards(N, old_tp)
            new_iv = shards(N, new_tp)
            old_h = {"w": [(ids[r], iv) for r, iv in enumerate(old_iv)]}
            new_h = {"w": [(ids[r], iv) for r, iv in enumerate(new_iv)]}
            plan = plan_transfers(old_h, new_h, valid_sources=set(ids), node_of={i: "n0" for i in ids})
            my_old = old_iv[rank] if rank < old_tp else (0, 0)
            my_new = new_iv[rank] if rank < new_tp else (0, 0)
            kinds = (("param", torch.bfloat16), ("exp_avg", torch.float32), ("exp_avg_sq", torch.float32))
            max_old = max(b - a for a, b in old_iv)
            max_new = max(b - a for a, b in new_iv)
            seg = {}
            for k, dt in kinds:
                seg[f"old_{k}"] = (max_old * N, dt)
                seg[f"new_{k}"] = (max_new * N, dt)
            heap = SymmetricHeap(seg, rank, world, exchange_via_group(), dev)
            g = torch.Generator(device=dev).manual_seed(0)
            full = {k: torch.empty(N, N, device=dev).normal_(generator=g).to(dt) for k, dt in kinds}
            for k, _ in kinds:
                t = heap.tensor(f"old_{k}")
                a, b = my_old
                if b > a:
                    t[: (b - a) * N].copy_(full[k][a:b].reshape(-1))
            torch.cuda.synchronize()
            dist.barrier()  # every old shard is in place before anyone pulls
            # pieces this rank pulls: (src, dst, bytes) for each kind
            triples = []
            esz = {k: torch.empty(0, dtype=dt).element_size() for k, dt in kinds}
            pieces = [(t.src, t.dst, t.interval) for t in plan.transfers] + [(d, d, iv) for d, _, iv in plan.reuse]
            for src_id, dst_id, (a, b) in pieces:
                if dst_id != ids[rank]:
                    continue
                src_rank = ids.index(src_id)
                o0, n0 = old_iv[src_rank][0], my_new[0]
                for k, _ in kinds:
                    src = heap.peer_ptrs(f"old_{k}")[src_rank] + (a - o0) * N * esz[k]
                    dst = heap.peer_ptrs(f"new_{k}")[rank] + (a - n0) * N * esz[k]
                    triples += [src, dst, (b - a) * N * esz[k]]
            lo_local, hi_local = heap.bases[rank], heap.bases[rank] + heap.nbytes
            remote_bytes = sum(triples[i + 2] for i in range(0, len(triples), 3)
                               if not lo_local <= triples[i] < hi_local)
            rb = torch.tensor([float(remote_bytes)], device=dev)
            dist.all_reduce(rb, op=dist.ReduceOp.MAX)

            def peer_once():
                ext().symm_copy(triples, dev.index)
                heap.barrier(30.0)

            def nccl_once():
                reqs = []
                for i, tr in enumerate(plan.transfers):
                    a, b = tr.interval
                    for j, (k, dt) in enumerate(kinds):
                        tag = i * 3 + j
                        if tr.src == ids[rank]:
                            o0 = my_old[0]
                            piece = heap.tensor(f"old_{k}")[(a - o0) * N:(b - o0) * N]
                            reqs.append(dist.isend(piece, ids.index(tr.dst), tag=tag))
                        if tr.dst == ids[rank]:
                            n0 = my_new[0]
                            buf = heap.tensor(f"new_{k}")[(a - n0) * N:(b - n0) * N]
                            reqs.append(dist.irecv(buf, ids.index(tr.src), tag=tag))
                for d, _, iv in plan.reuse:
                    if d == ids[rank]:
                        a, b = iv
                        for k, _ in kinds:
                            heap.tensor(f"new_{k}")[(a - my_new[0]) * N:(b - my_new[0]) * N].copy_(
                                heap.tensor(f"old_{k}")[(a - my_old[0]) * N:(b - my_old[0]) * N])
                for r in reqs:
                    r.wait()

            for impl, fn in (("peer", peer_once), ("nccl", nccl_once)):
                for _ in range(2):
                    fn()
                torch.cuda.synchronize()
                times = []
                for _ in range(iters):
                    dist.barrier()
                    torch.cuda.synchronize()
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    fn()
                    e.record()
                    torch.cuda.synchronize()
                    times.append(s.elapsed_time(e))
                t = torch.tensor([sorted(times)[len(times) // 2]], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
                # correctness: the new shard equals the slice of the full tensors
                ok = True
                a, b = my_new
                if b > a:
                    for k, _ in kinds:
                        ok &= bool(torch.equal(heap.tensor(f"new_{k}")[: (b - a) * N].view(b - a, N), full[k][a:b]))
                okt = torch.tensor([1.0 if ok else 0.0], device=dev)
                dist.all_reduce(okt, op=dist.ReduceOp.MIN)
                roof_ms = float(rb.item()) / (NVLINK_GBS * 1e9) * 1e3
                row = {"N": N, "transition": f"TP{old_tp}->TP{new_tp}", "impl": impl, "ms": round(ms, 4),
                       "busiest_rank_remote_MB": round(float(rb.item()) / 1e6, 1),
                       "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3),
                       "exact": bool(okt.item() == 1.0)}
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
                for k, _ in kinds:
                    heap.tensor(f"new_{k}").zero_()
            torch.cuda.synchronize()
            dist.barrier()
            heap.close()
            del full
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes", default="4096,8192,16384")
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    run(tuple(int(x) for x in a.sizes.split(",")), a.iters)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
