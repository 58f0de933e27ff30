"""Validation probes that pinpoint a slow GPU or link after a confirmed change point.

* compute: a short GEMM benchmark per suspect device against its healthy reference -- on
  B200 through this package's own tcgen05 GEMM (``ops.gemm``), elsewhere ``torch.matmul``;
* links: point-to-point bandwidth probes in O(max degree) rounds of disjoint pairs (greedy edge
  colouring: 2 rounds for an even ring, 3 for an odd one), so the fabric is checked in a constant
  number of steps at any scale.
(Reference: ``resihp/detect/validation.py:17-84``.)
"""

from __future__ import annotations

import time

import torch
import torch.distributed as dist


def gemm_tflops(n: int = 2048, iters: int = 10, device: str | None = None, dtype: torch.dtype | None = None,
                use_native: bool = True) -> float:
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    dtype = dtype or (torch.bfloat16 if dev.type == "cuda" else torch.float32)
    a = torch.randn(n, n, device=dev, dtype=dtype)
    b = torch.randn(n, n, device=dev, dtype=dtype)
    if dev.type == "cuda" and use_native and dtype == torch.bfloat16:
        from ..ops import gemm

        out = torch.empty(n, n, device=dev, dtype=dtype)

        def mm():
            gemm(a, b, out=out)
    else:
        def mm():
            a @ b
    for _ in range(2):
        mm()
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            mm()
        e.record()
        torch.cuda.synchronize(dev)
        secs = s.elapsed_time(e) / 1e3
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            mm()
        secs = time.perf_counter() - t0
    return 2 * n ** 3 * iters / secs / 1e12


def slowdown_vs_reference(measured: float, reference: float) -> float:
    """> 1 means slower than the device's healthy reference."""
    return reference / max(measured, 1e-12)


def edge_rounds(edges: list[tuple[int, int]]) -> list[list[tuple[int, int]]]:
    """Greedy edge colouring: every round is a set of disjoint links probed concurrently."""
    rounds: list[tuple[set[int], list[tuple[int, int]]]] = []
    for a, b in sorted(edges, key=lambda e: (min(e), max(e))):
        for used, rnd in rounds:
            if a not in used and b not in used:
                rnd.append((a, b))
                used.update((a, b))
                break
        else:
            rounds.append(({a, b}, [(a, b)]))
    return [rnd for _, rnd in rounds]


def ring_edges(order: list[int]) -> list[tuple[int, int]]:
    n = len(order)
    if n < 2:
        return []
    if n == 2:
        return [(order[0], order[1])]
    return [(order[i], order[(i + 1) % n]) for i in range(n)]


def probe_links(rank: int, rounds: list[list[tuple[int, int]]], mgr, nbytes: int = 8 << 20, repeats: int = 3,
                timeout: float = 60.0, device: str = "cpu") -> dict[tuple[int, int], float]:
    """GB/s of each link this rank belongs to (``rounds`` must be identical on every rank)."""
    buf = torch.empty(nbytes // 4, dtype=torch.float32, device=device)
    out = {}
    for rnd in rounds:
        for a, b in rnd:
            if rank not in (a, b):
                continue
            peer = b if rank == a else a
            t0 = time.perf_counter()
            for i in range(repeats):
                first, second = (dist.isend, dist.irecv) if rank == a else (dist.irecv, dist.isend)
                mgr.guarded_wait(first(buf, peer, tag=7000 + i), timeout=timeout, what="link probe")
                mgr.guarded_wait(second(buf, peer, tag=8000 + i), timeout=timeout, what="link probe")
            out[(a, b)] = 2 * repeats * nbytes / (time.perf_counter() - t0) / 1e9
    return out
