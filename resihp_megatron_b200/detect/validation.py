"""Validation probes that pinpoint the slow GPU or link after a confirmed change point.

* **Compute**: a short GEMM benchmark on a suspect device, compared with its healthy reference.
  On B200 it runs this package's own tcgen05 GEMM (``ops.gemm``) -- the kernel the training
  step uses -- elsewhere ``torch.matmul``.
* **Links**: point-to-point bandwidth in O(max degree) rounds of disjoint pairs (a greedy edge
  colouring: 2 rounds for an even ring, 3 for an odd one), so the fabric is checked in a
  constant number of steps at any scale.  ``probe_links`` measures the NCCL (SM-driven) path
  between ranks; ``copy_engine_gbps`` measures a copy-engine peer copy between two GPUs of this
  process.
Parity: ``resihp/detect/validation.py:17-84`` (same probes; the GEMM is ours, not cuBLAS).
"""

from __future__ import annotations

import time
from typing import Callable

import torch
import torch.distributed as dist


def _seconds(fn: Callable[[], None], iters: int, device: torch.device) -> float:
    """Wall time of ``iters`` calls, with CUDA events on a GPU (after two untimed calls)."""
    fn()
    fn()
    if device.type != "cuda":
        started = time.perf_counter()
        for _ in range(iters):
            fn()
        return time.perf_counter() - started
    torch.cuda.synchronize(device)
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize(device)
    return begin.elapsed_time(end) / 1000.0


def gemm_tflops(n: int = 2048, iters: int = 10, device: str | None = None, dtype: torch.dtype | None = None,
                use_native: bool = True) -> float:
    """TFLOP/s of an ``n x n x n`` GEMM (this package's tcgen05 kernel on CUDA in bf16)."""
    dev = torch.device(device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu"))
    dtype = dtype or (torch.bfloat16 if dev.type == "cuda" else torch.float32)
    lhs, rhs = (torch.randn(n, n, device=dev, dtype=dtype) for _ in range(2))
    if dev.type == "cuda" and use_native and dtype == torch.bfloat16:
        from ..ops import gemm

        product = torch.empty(n, n, device=dev, dtype=dtype)
        secs = _seconds(lambda: gemm(lhs, rhs, out=product), iters, dev)
    else:
        secs = _seconds(lambda: lhs @ rhs, iters, dev)
    return 2.0 * n ** 3 * iters / secs / 1e12


def slowdown_vs_reference(measured: float, reference: float) -> float:
    """> 1 means slower than the device's healthy reference."""
    return reference / max(measured, 1e-12)


def copy_engine_gbps(src: int, dst: int, nbytes: int = 256 << 20, iters: int = 5) -> float:
    """GB/s of a peer copy from GPU ``src`` to GPU ``dst`` (copy engines over NVLink)."""
    a = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{src}")
    b = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dst}")
    with torch.cuda.device(src):
        secs = _seconds(lambda: b.copy_(a, non_blocking=True), iters, torch.device("cuda", src))
    return nbytes * iters / secs / 1e9


def edge_rounds(edges: list[tuple[int, int]]) -> list[list[tuple[int, int]]]:
    """Greedy edge colouring: each round is a set of vertex-disjoint links probed together."""
    busy: list[set[int]] = []   # per round, the vertices it already uses
    rounds: list[list[tuple[int, int]]] = []
    for a, b in sorted(edges, key=lambda e: tuple(sorted(e))):
        k = next((i for i, used in enumerate(busy) if a not in used and b not in used), len(rounds))
        if k == len(rounds):
            busy.append(set())
            rounds.append([])
        busy[k] |= {a, b}
        rounds[k].append((a, b))
    return rounds


def ring_edges(order: list[int]) -> list[tuple[int, int]]:
    """Links of a ring over ``order`` (one link for two members, none for fewer)."""
    n = len(order)
    if n <= 2:
        return [tuple(order)] if n == 2 else []
    return list(zip(order, order[1:] + order[:1]))


def probe_links(rank: int, rounds: list[list[tuple[int, int]]], mgr, nbytes: int = 8 << 20, repeats: int = 3,
                timeout: float = 60.0, device: str = "cpu") -> dict[tuple[int, int], float]:
    """GB/s of every link this rank is on (``rounds`` must be the same on every rank): each
    repeat sends one way, then the other, through the generation's communicator."""
    payload = torch.empty(nbytes // 4, dtype=torch.float32, device=device)
    measured = {}
    for a, b in (link for rnd in rounds for link in rnd if rank in link):
        peer, leads = (b, True) if rank == a else (a, False)
        started = time.perf_counter()
        for i in range(repeats):
            legs = (dist.isend, dist.irecv) if leads else (dist.irecv, dist.isend)
            for leg, tag in zip(legs, (7000 + i, 8000 + i)):
                mgr.guarded_wait(leg(payload, peer, tag=tag), timeout=timeout, what="link probe")
        measured[(a, b)] = 2 * repeats * nbytes / (time.perf_counter() - started) / 1e9
    return measured
