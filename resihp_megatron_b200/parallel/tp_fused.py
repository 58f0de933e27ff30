"""Tensor-parallel layers with the collective fused into the GEMM, on symmetric peer memory.

* ``all_gather_gemm`` -- column-parallel layer with sequence-parallel input:
  ``Y[M, N_local] = AllGather_rows(X)[M, K] @ W_local[N_local, K]^T``.  Each rank writes its
  ``[M / tp, K]`` token shard into its own chunk of a heap-resident gather buffer; after a bounded
  barrier one cooperative kernel pulls the peers' chunks over NVLink with dedicated copy warps
  while its MMA warps already multiply the chunks that have landed (own chunk first).
  Replaces reference call site C2 (``resihp/runtime/reference_model.py:173-181``: all-gather then
  ``F.linear``).
* ``gemm_reduce_scatter`` -- row-parallel layer with sequence-parallel output:
  ``Y_local[M / tp, N] = sum_r (X_r[M, K_local] @ W_r[N, K_local]^T)[rows of this rank]``.  The GEMM
  epilogue stores each bf16 partial tile straight into the owning rank's receive slot over NVLink;
  after a bounded barrier every rank sums its slots in rank order (fp32 accumulate, deterministic).
  Replaces C3 (``reference_model.py:147-149,184-192``: all-reduce + narrow).

Both need M divisible by tp (and the gather chunk by 128 rows).  No TMA ever reads peer memory
here: the copy warps use plain 16-byte loads, and the GEMM's TMA reads only this rank's buffers.
"""

from __future__ import annotations

import torch

from ..ops._build import ext
from ..ops.counter import count
from .symm import AbortWord, SymmetricHeap


class TensorParallelComm:
    def __init__(self, rank: int, world: int, exchange, device, *, max_rows: int, max_k: int, max_n: int,
                 abort: AbortWord | None = None, budget_s: float = 30.0, _heap: SymmetricHeap | None = None):
        self.rank, self.world = rank, world
        self.max_rows, self.max_k, self.max_n = max_rows, max_k, max_n
        self.abort = abort
        self.budget = budget_s
        segs = {"x_full": (max_rows * max_k, torch.bfloat16),
                "rs_recv": (world * (max_rows // world) * max_n, torch.bfloat16)}
        self.heap = _heap or SymmetricHeap(segs, rank, world, exchange, device, abort)
        self.ready = torch.zeros(world, dtype=torch.int32, device=device)
        self.emulated = _heap is not None

    @classmethod
    def emulated_group(cls, world: int, device, **kw) -> list["TensorParallelComm"]:
        """``world`` ranks in one process on one GPU (tests): call the per-rank steps in turn."""
        segs = {"x_full": (kw["max_rows"] * kw["max_k"], torch.bfloat16),
                "rs_recv": (world * (kw["max_rows"] // world) * kw["max_n"], torch.bfloat16)}
        heaps = SymmetricHeap.emulated(segs, world, device)
        return [cls(r, world, None, device, _heap=heaps[r], **kw) for r in range(world)]

    def _barrier(self) -> None:
        if not self.emulated:
            self.heap.barrier(self.budget)

    # ------------------------------------------------------------------ all-gather -> GEMM
    def gather_buffer(self, M: int, K: int) -> torch.Tensor:
        return self.heap.tensor("x_full")[: M * K].view(M, K)

    def local_chunk(self, M: int, K: int) -> torch.Tensor:
        """Where this rank writes its ``[M / tp, K]`` shard before ``all_gather_gemm``."""
        rows = M // self.world
        return self.gather_buffer(M, K)[self.rank * rows:(self.rank + 1) * rows]

    def all_gather_gemm(self, M: int, w: torch.Tensor, out: torch.Tensor | None = None,
                        finish: bool = True) -> torch.Tensor:
        K = w.shape[1]
        rows = M // self.world
        xf = self.gather_buffer(M, K)
        y = torch.empty(M, w.shape[0], dtype=torch.bfloat16, device=w.device) if out is None else out
        base = self.heap.peer_ptrs("x_full")
        src = [base[c] + c * rows * K * 2 for c in range(self.world)]
        self._barrier()  # every rank's chunk is in place
        ext().tp_ag_gemm(xf, src, self.rank, w, y, self.ready, self.abort.dev if self.abort else 0)
        if finish:
            self._barrier()  # nobody still reads this rank's chunk
        count(3 if not self.emulated else 1)
        return y

    # ------------------------------------------------------------------ GEMM -> reduce-scatter
    def gemm_reduce_scatter(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Emulated groups: call ``scatter_partials`` on every rank, then ``reduce_received``."""
        self._barrier()  # receive slots are free again
        self.scatter_partials(x, w)
        self._barrier()  # every partial has landed
        return self.reduce_received(x.shape[0], w.shape[0], out)

    def scatter_partials(self, x: torch.Tensor, w: torch.Tensor) -> None:
        ext().tp_rs_gemm(x, w, self.heap.peer_ptrs("rs_recv"), self.rank)
        count(1)

    def reduce_received(self, M: int, N: int, out: torch.Tensor | None = None) -> torch.Tensor:
        rows = M // self.world
        y = torch.empty(rows, N, dtype=torch.bfloat16, device=self.ready.device) if out is None else out
        ext().tp_rs_reduce(self.heap.tensor("rs_recv")[: self.world * rows * N], self.world, y)
        count(1)
        return y

    def close(self) -> None:
        if not self.emulated or self.rank == 0:
            self.heap.close()
