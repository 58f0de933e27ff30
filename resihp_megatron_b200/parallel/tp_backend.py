"""Tensor-parallel collectives of a sequence-parallel transformer stage behind one interface.

A stage with sequence parallelism keeps the residual stream sharded by token rows (``M`` rows of
a micro-batch split evenly over the ``tp`` ranks); around every column-parallel GEMM the rows are
all-gathered, after every row-parallel GEMM the partial products are reduce-scattered back to
the row shards.  Three implementations:

* ``FusedTP`` -- the collectives fused into the GEMMs on symmetric NVLink peer memory
  (``TensorParallelComm``: one persistent all-gather -> GEMM kernel; a GEMM whose epilogue stores
  the partial tiles into their owners' receive slots, then a rank-ordered reduce);
* ``CollectiveTP`` -- ``torch.distributed`` all-gather / reduce-scatter around the same GEMM
  kernel (NCCL on GPUs, gloo on CPU): the baseline the fused path is measured against;
* ``SoloTP`` -- one rank, no communication.

Operations:

* ``chunk(M, K)`` -- the ``[M / tp, K]`` rows this rank contributes to the next gather; the
  producer (an RMSNorm, a copy) writes them in place;
* ``ag_gemm(M, w, out, w_t)`` -> ``(AllGather(chunks) @ op(w)^T, gathered input)``;
* ``all_gather(M, K)`` -> the gathered ``[M, K]`` chunks;
* ``gemm_rs(x, w, out, w_t, residual)`` -> ``ReduceScatter_rows(x @ op(w)^T) (+ residual)``;
* ``fp8_local(M, K)`` / ``all_gather_fp8(M, K)`` -- the gather of a block-scaled fp8 input: this
  rank quantises its rows (1 x 128 row scales, row-major so a row's scales travel with it) into
  ``fp8_local``'s ``(data [M / tp, K] uint8, scales [M / tp, K / 128])``; the gather returns the
  ``[M, K]`` / ``[M, K / 128]`` views -- half the bytes of the bf16 gather, and no
  quantisation pass over the gathered rows;
* ``gemm_rs_with(M, N, gemm, out, residual)`` -> the same for any GEMM (the block-scaled fp8
  one): ``gemm(out=..., residual=..., scatter=(recv_ptrs, slot))`` writes the ``[M, N]`` product
  into a local buffer (optionally plus a residual) or, with ``scatter``, stores each row
  straight into its owner's receive slot.

``op(w) = w`` (``[N, K]``) or, with ``w_t``, ``w.T`` (``w`` stored ``[K, N]``).  A gathered input
stays valid until the gather after next (two buffers alternate), which is what the weight
gradients of a layer need.  (Reference: the sequence-parallel autograd functions
``_GatherFromSP`` / ``_ReduceScatterToSP``, ``resihp/runtime/reference_model.py:134-192``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops


class _Buffers:
    """Two alternating ``[M, K]`` bf16 buffers per shape."""

    def __init__(self, device):
        self.device = device
        self.bufs: dict[tuple[int, int], list[torch.Tensor]] = {}
        self.turn = 0

    def current(self, M: int, K: int) -> torch.Tensor:
        pair = self.bufs.get((M, K))
        if pair is None:
            pair = [torch.empty(M, K, dtype=torch.bfloat16, device=self.device) for _ in range(2)]
            self.bufs[(M, K)] = pair
        return pair[self.turn]

    def advance(self) -> None:
        self.turn ^= 1


class _Fp8Buffers:
    """Two alternating ``([M, K] uint8, [M, K / 128] fp32)`` buffers per shape."""

    def __init__(self, device):
        self.device = device
        self.bufs: dict[tuple[int, int], list] = {}
        self.turn = 0

    def current(self, M: int, K: int):
        pair = self.bufs.get((M, K))
        if pair is None:
            pair = [(torch.empty(M, K, dtype=torch.uint8, device=self.device),
                     torch.empty(M, K // 128, dtype=torch.float32, device=self.device)) for _ in range(2)]
            self.bufs[(M, K)] = pair
        return pair[self.turn]

    def advance(self) -> None:
        self.turn ^= 1


class SoloTP:
    world, rank = 1, 0

    def __init__(self, device):
        self.buf = _Buffers(device)
        self.f8 = _Fp8Buffers(device)

    def fp8_local(self, M: int, K: int):
        return self.f8.current(M, K)

    def all_gather_fp8(self, M: int, K: int):
        out = self.f8.current(M, K)
        self.f8.advance()
        return out

    def chunk(self, M: int, K: int) -> torch.Tensor:
        return self.buf.current(M, K)

    def ag_gemm(self, M: int, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False):
        K = w.shape[0] if w_t else w.shape[1]
        x = self.buf.current(M, K)
        self.buf.advance()
        return ops.gemm(x, w, b_t=w_t, out=out), x

    def all_gather(self, M: int, K: int) -> torch.Tensor:
        x = self.buf.current(M, K)
        self.buf.advance()
        return x

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        return ops.gemm(x, w, b_t=w_t, out=out, residual=residual)

    def gemm_rs_with(self, M: int, N: int, gemm, out: torch.Tensor | None = None,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
        return gemm(out=out, residual=residual)

    def close(self) -> None:
        pass


class CollectiveTP:
    """Library collectives on ``group`` (this rank is ``rank`` of ``world``)."""

    def __init__(self, rank: int, world: int, group, device, waiter=None):
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.buf = _Buffers(self.device)
        self.f8 = _Fp8Buffers(self.device)
        self.partials: dict[tuple[int, int], torch.Tensor] = {}
        self.wait = waiter or (lambda work: work.wait())

    def chunk(self, M: int, K: int) -> torch.Tensor:
        rows = M // self.world
        return self.buf.current(M, K)[self.rank * rows:(self.rank + 1) * rows]

    def fp8_local(self, M: int, K: int):
        q, s = self.f8.current(M, K)
        rows = M // self.world
        return q[self.rank * rows:(self.rank + 1) * rows], s[self.rank * rows:(self.rank + 1) * rows]

    def all_gather_fp8(self, M: int, K: int):
        q, s = self.f8.current(M, K)
        self.f8.advance()
        ql, sl = q.chunk(self.world)[self.rank], s.chunk(self.world)[self.rank]
        self.wait(dist.all_gather_into_tensor(q, ql, group=self.group, async_op=True))
        self.wait(dist.all_gather_into_tensor(s, sl, group=self.group, async_op=True))
        return q, s

    def all_gather(self, M: int, K: int) -> torch.Tensor:
        full = self.buf.current(M, K)
        self.buf.advance()
        rows = M // self.world
        mine = full[self.rank * rows:(self.rank + 1) * rows]
        self.wait(dist.all_gather_into_tensor(full, mine, group=self.group, async_op=True))
        return full

    def ag_gemm(self, M: int, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False):
        K = w.shape[0] if w_t else w.shape[1]
        x = self.all_gather(M, K)
        return ops.gemm(x, w, b_t=w_t, out=out), x

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        M, N = x.shape[0], (w.shape[1] if w_t else w.shape[0])
        part = self.partials.get((M, N))
        if part is None:
            part = self.partials[(M, N)] = torch.empty(M, N, dtype=torch.bfloat16, device=self.device)
        ops.gemm(x, w, b_t=w_t, out=part)
        return self._reduce_scatter(part, out, residual)

    def gemm_rs_with(self, M: int, N: int, gemm, out: torch.Tensor | None = None,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
        part = self.partials.get((M, N))
        if part is None:
            part = self.partials[(M, N)] = torch.empty(M, N, dtype=torch.bfloat16, device=self.device)
        gemm(out=part)
        return self._reduce_scatter(part, out, residual)

    def _reduce_scatter(self, part: torch.Tensor, out, residual) -> torch.Tensor:
        M, N = part.shape
        y = torch.empty(M // self.world, N, dtype=torch.bfloat16, device=self.device) if out is None else out
        self.wait(dist.reduce_scatter_tensor(y, part, group=self.group, async_op=True))
        if residual is not None:
            y.add_(residual)
        return y

    def close(self) -> None:
        pass


class FusedTP:
    """``TensorParallelComm`` (symmetric heap of this TP group) behind the stage interface."""

    def __init__(self, comm):
        self.comm = comm
        self.rank, self.world = comm.rank, comm.world

    def chunk(self, M: int, K: int) -> torch.Tensor:
        return self.comm.local_chunk(M, K)

    def ag_gemm(self, M: int, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False):
        K = w.shape[0] if w_t else w.shape[1]
        x = self.comm.gather_buffer(M, K)
        return self.comm.all_gather_gemm(M, w, out=out, w_t=w_t), x

    def all_gather(self, M: int, K: int) -> torch.Tensor:
        return self.comm.all_gather(M, K)

    def fp8_local(self, M: int, K: int):
        return self.comm.fp8_local(M, K)

    def all_gather_fp8(self, M: int, K: int):
        return self.comm.all_gather_fp8(M, K)

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        return self.comm.gemm_reduce_scatter(x, w, out=out, w_t=w_t, residual=residual)

    def gemm_rs_with(self, M: int, N: int, gemm, out: torch.Tensor | None = None,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
        return self.comm.reduce_scatter_with(M, N, gemm, out=out, residual=residual)

    def check(self) -> None:
        self.comm.heap.check()

    def close(self) -> None:
        self.comm.close()
