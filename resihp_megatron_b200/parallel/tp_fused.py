"""Tensor-parallel layers with the collective fused into the GEMM, on symmetric peer memory.

* ``all_gather_gemm`` -- column-parallel layer with sequence-parallel input:
  ``Y[M, N_local] = AllGather_rows(X)[M, K] @ W_local[N_local, K]^T``.  Each rank writes its
  ``[M / tp, K]`` token shard into its own chunk of a heap-resident gather buffer; after a bounded
  barrier one persistent kernel pulls the peers' chunks over NVLink with dedicated copy warps
  (128-row x 512-column units claimed from a work counter, each published by a flag) while its
  MMA warps already multiply the units that have landed (own chunk first).
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
    """Per tensor-parallel group: two gather buffers and two reduce-scatter receive buffers in the
    symmetric heap, used alternately.  Every collective starts with a bounded barrier; since a
    buffer is reused only two collectives later, that leading barrier (which each rank reaches
    after finishing its previous kernels) already guarantees nobody still reads it, so no trailing
    barrier is needed."""

    def __init__(self, rank: int, world: int, exchange, device, *, max_rows: int, max_k: int, max_n: int,
                 abort: AbortWord | None = None, budget_s: float = 30.0, _heap: SymmetricHeap | None = None):
        self.rank, self.world = rank, world
        self.max_rows, self.max_k, self.max_n = max_rows, max_k, max_n
        self.abort = abort
        self.budget = budget_s
        self.heap = _heap or SymmetricHeap(self.segments(world, max_rows, max_k, max_n), rank, world, exchange,
                                           device, abort)
        # work counter + one flag per copy unit of the all-gather -> GEMM kernel
        self.ready = torch.zeros(1 + (max_rows // 128) * (-(-max_k // 512)), dtype=torch.int32, device=device)
        self.emulated = _heap is not None
        self._ag = 0
        self._rs = 0

    @staticmethod
    def segments(world: int, max_rows: int, max_k: int, max_n: int) -> dict:
        return {"x_full0": (max_rows * max_k, torch.bfloat16), "x_full1": (max_rows * max_k, torch.bfloat16),
                "rs_recv0": (world * (max_rows // world) * max_n, torch.bfloat16),
                "rs_recv1": (world * (max_rows // world) * max_n, torch.bfloat16)}

    @classmethod
    def emulated_group(cls, world: int, device, **kw) -> list["TensorParallelComm"]:
        """``world`` ranks in one process on one GPU (tests): call the per-rank steps in turn."""
        heaps = SymmetricHeap.emulated(cls.segments(world, kw["max_rows"], kw["max_k"], kw["max_n"]), world, device)
        return [cls(r, world, None, device, _heap=heaps[r], **kw) for r in range(world)]

    def _barrier(self) -> None:
        if not self.emulated:
            self.heap.barrier(self.budget)

    # ------------------------------------------------------------------ all-gather (-> GEMM)
    def gather_buffer(self, M: int, K: int, buf: int | None = None) -> torch.Tensor:
        b = self._ag if buf is None else buf
        return self.heap.tensor(f"x_full{b}")[: M * K].view(M, K)

    def advance_gather(self) -> None:
        """Use the other gather buffer next (a gather that moved nothing still takes its turn)."""
        self._ag ^= 1

    def local_chunk(self, M: int, K: int) -> torch.Tensor:
        """Where this rank writes its ``[M / tp, K]`` shard before the next gather."""
        rows = M // self.world
        return self.gather_buffer(M, K)[self.rank * rows:(self.rank + 1) * rows]

    def _sources(self, M: int, K: int, b: int) -> list[int]:
        rows = M // self.world
        base = self.heap.peer_ptrs(f"x_full{b}")
        return [base[c] + c * rows * K * 2 for c in range(self.world)]

    def all_gather_gemm(self, M: int, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False,
                        advance: bool = True) -> torch.Tensor:
        """``AllGather(chunks)[M, K] @ op(w)^T`` with ``op(w) = w`` ([N, K]) or ``w.T`` (``w_t``,
        ``w`` is [K, N]).  The gathered input stays in the gather buffer until the buffer's next
        use (two gathers later) -- weight gradients read it from there."""
        K = w.shape[0] if w_t else w.shape[1]
        N = w.shape[1] if w_t else w.shape[0]
        b = self._ag
        xf = self.gather_buffer(M, K, b)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=w.device) if out is None else out
        self._barrier()  # every rank's chunk is in place; the buffer's previous readers are done
        ext().tp_ag_gemm(xf, self._sources(M, K, b), self.rank, w, bool(w_t), y, self.ready,
                         self.abort.dev if self.abort else 0)
        count(2 if not self.emulated else 1)
        if advance:
            self._ag ^= 1
        return y

    def all_gather(self, M: int, K: int, advance: bool = True) -> torch.Tensor:
        """Plain all-gather of the chunks (peer pulls); returns the gathered ``[M, K]`` view."""
        b = self._ag
        xf = self.gather_buffer(M, K, b)
        rows = M // self.world
        self._barrier()
        ext().symm_gather(self._sources(M, K, b), self.heap.peer_ptrs(f"x_full{b}")[self.rank], rows * K * 2,
                          self.rank, xf.device.index if xf.device.index is not None else 0)
        count(2 if not self.emulated else 1)
        if advance:
            self._ag ^= 1
        return xf

    # ------------------------------------------------------------------ fp8 all-gather
    def _fp8_offset(self, M: int, K: int) -> int:
        return (M * K + 255) // 256 * 256

    def fp8_views(self, M: int, K: int, buf: int | None = None):
        """The fp8 gather layout inside gather buffer ``buf``: ``[M, K]`` bytes, then row-major
        ``[M, K / 128]`` fp32 scales (together at most half the bf16 ``[M, K]`` buffer + M K / 32)."""
        b = self._ag if buf is None else buf
        raw = self.heap.tensor(f"x_full{b}").view(torch.uint8)
        off, nk = self._fp8_offset(M, K), K // 128
        assert off + M * nk * 4 <= raw.numel(), "fp8 gather does not fit the gather buffer"
        return raw[: M * K].view(M, K), raw[off: off + M * nk * 4].view(torch.float32).view(M, nk)

    def fp8_local(self, M: int, K: int):
        """Where this rank quantises its ``[M / tp, K]`` rows (and their scales) before the gather."""
        q, s = self.fp8_views(M, K)
        rows = M // self.world
        return q[self.rank * rows:(self.rank + 1) * rows], s[self.rank * rows:(self.rank + 1) * rows]

    def all_gather_fp8(self, M: int, K: int, advance: bool = True):
        """Gather every rank's fp8 rows and row scales (peer pulls, two launches)."""
        b = self._ag
        q, s = self.fp8_views(M, K, b)
        rows, nk = M // self.world, K // 128
        off = self._fp8_offset(M, K)
        if (rows * K) % 16 or (rows * nk * 4) % 16:
            raise ValueError("fp8 gather chunks must be multiples of 16 bytes")
        base = self.heap.peer_ptrs(f"x_full{b}")
        dev = q.device.index if q.device.index is not None else 0
        self._barrier()
        ext().symm_gather([base[c] + c * rows * K for c in range(self.world)], base[self.rank], rows * K, self.rank,
                          dev)
        ext().symm_gather([base[c] + off + c * rows * nk * 4 for c in range(self.world)], base[self.rank] + off,
                          rows * nk * 4, self.rank, dev)
        count(3 if not self.emulated else 2)
        if advance:
            self._ag ^= 1
        return q, s

    # ------------------------------------------------------------------ GEMM -> reduce-scatter
    def gemm_reduce_scatter(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
                            w_t: bool = False, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``ReduceScatter_rows(x @ op(w)^T)`` (+ ``residual``, this rank's rows).  Emulated groups:
        call ``scatter_partials`` on every rank, then ``reduce_received``."""
        self._barrier()  # receive slots of this buffer are free again
        self.scatter_partials(x, w, w_t)
        self._barrier()  # every partial has landed
        y = self.reduce_received(x.shape[0], w.shape[1] if w_t else w.shape[0], out, residual)
        self._rs ^= 1
        return y

    def gemm_reduce_scatter_begin(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, w_t: bool = False):
        """``gemm_reduce_scatter`` in two halves: the partials are scattered now; the returned
        ``finish()`` waits (bounded barrier) for every rank's partials and reduces them into
        ``out``.  Work enqueued before ``finish()`` runs while the peers catch up."""
        self._barrier()
        self.scatter_partials(x, w, w_t)
        M, N = x.shape[0], (w.shape[1] if w_t else w.shape[0])

        def finish() -> None:
            self._barrier()
            self.reduce_received(M, N, out, None)
            self._rs ^= 1

        return finish

    def reduce_scatter_with(self, M: int, N: int, gemm, out: torch.Tensor | None = None,
                            residual: torch.Tensor | None = None) -> torch.Tensor:
        """``gemm_reduce_scatter`` for another GEMM kernel (the block-scaled fp8 one) whose
        epilogue stores row ``m`` into rank ``m // (M / world)``'s receive slot:
        ``gemm(scatter=(recv_ptrs, slot))``."""
        self._barrier()
        gemm(scatter=(self.heap.peer_ptrs(f"rs_recv{self._rs}"), self.rank))
        self._barrier()
        y = self.reduce_received(M, N, out, residual)
        self._rs ^= 1
        return y

    def scatter_partials(self, x: torch.Tensor, w: torch.Tensor, w_t: bool = False) -> None:
        ext().tp_rs_gemm(x, w, bool(w_t), self.heap.peer_ptrs(f"rs_recv{self._rs}"), self.rank)
        count(1)

    def reduce_received(self, M: int, N: int, out: torch.Tensor | None = None,
                        residual: torch.Tensor | None = None) -> torch.Tensor:
        rows = M // self.world
        y = torch.empty(rows, N, dtype=torch.bfloat16, device=self.ready.device) if out is None else out
        ext().tp_rs_reduce(self.heap.tensor(f"rs_recv{self._rs}")[: self.world * rows * N], self.world, y, residual)
        count(1)
        return y

    def close(self) -> None:
        if not self.emulated or self.rank == 0:
            self.heap.close()
