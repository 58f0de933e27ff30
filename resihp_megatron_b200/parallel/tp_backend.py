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
* ``gemm_rs_async(x, w, out, w_t)`` -> a ``finish()`` callable: the GEMM and the start of the
  reduce-scatter are enqueued now, ``out`` holds the reduced rows once ``finish()`` returned, and
  work enqueued in between (a weight-gradient GEMM) overlaps the transfer;
* ``fp8_local(M, K)`` / ``all_gather_fp8(M, K)`` -- the gather of a block-scaled fp8 input: this
  rank quantises its rows (1 x 128 row scales, row-major so a row's scales travel with it) into
  ``fp8_local``'s ``(data [M / tp, K] uint8, scales [M / tp, K / 128])``; the gather returns the
  ``[M, K]`` / ``[M, K / 128]`` views -- half the bytes of the bf16 gather, and no
  quantisation pass over the gathered rows;
* ``gemm_rs_with(M, N, gemm, out, residual)`` -> the same for any GEMM (the block-scaled fp8
  one): ``gemm(out=..., residual=..., scatter=(recv_ptrs, slot))`` writes the ``[M, N]`` product
  into a local buffer (optionally plus a residual) or, with ``scatter``, stores each row
  straight into its owner's receive slot.

``op(w) = w`` (``[N, K]``) or, with ``w_t``, ``w.T`` (``w`` stored ``[K, N]``).

Without sequence parallelism (``sp=False``) the residual stream is replicated on every TP rank:
``chunk`` is the whole ``[M, K]`` buffer, the gathers move nothing, and the reduce-scatter
becomes an all-reduce (the GEMM -> all-reduce of Megatron's plain tensor parallelism; fused:
the GEMM -> reduce-scatter kernel pair followed by a peer all-gather of the reduced rows).  A gathered input
stays valid until the gather after next (two buffers alternate), which is what the weight
gradients of a layer need.  (Reference: the sequence-parallel autograd functions
``_GatherFromSP`` / ``_ReduceScatterToSP``, ``resihp/runtime/reference_model.py:134-192``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops


def _done() -> None:
    pass


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
    sp = True  # one rank: both modes coincide

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

    def gemm_rs_async(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, w_t: bool = False):
        self.gemm_rs(x, w, out=out, w_t=w_t)
        return _done

    def close(self) -> None:
        pass


class CollectiveTP:
    """Library collectives on ``group`` (this rank is ``rank`` of ``world``)."""

    def __init__(self, rank: int, world: int, group, device, waiter=None, sp: bool = True):
        self.rank, self.world, self.group = rank, world, group
        self.sp = sp
        self.device = torch.device(device)
        self.buf = _Buffers(self.device)
        self.f8 = _Fp8Buffers(self.device)
        self.partials: dict[tuple[int, int], torch.Tensor] = {}
        self.wait = waiter or (lambda work: work.wait())

    def chunk(self, M: int, K: int) -> torch.Tensor:
        if not self.sp:
            return self.buf.current(M, K)
        rows = M // self.world
        return self.buf.current(M, K)[self.rank * rows:(self.rank + 1) * rows]

    def fp8_local(self, M: int, K: int):
        q, s = self.f8.current(M, K)
        if not self.sp:
            return q, s
        rows = M // self.world
        return q[self.rank * rows:(self.rank + 1) * rows], s[self.rank * rows:(self.rank + 1) * rows]

    def all_gather_fp8(self, M: int, K: int):
        q, s = self.f8.current(M, K)
        self.f8.advance()
        if not self.sp:
            return q, s
        ql, sl = q.chunk(self.world)[self.rank], s.chunk(self.world)[self.rank]
        self.wait(dist.all_gather_into_tensor(q, ql, group=self.group, async_op=True))
        self.wait(dist.all_gather_into_tensor(s, sl, group=self.group, async_op=True))
        return q, s

    def all_gather(self, M: int, K: int) -> torch.Tensor:
        full = self.buf.current(M, K)
        self.buf.advance()
        if not self.sp:
            return full
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

    def gemm_rs_async(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, w_t: bool = False):
        if not self.sp:
            self.gemm_rs(x, w, out=out, w_t=w_t)
            return _done
        M, N = x.shape[0], (w.shape[1] if w_t else w.shape[0])
        part = self.partials.get((M, N))
        if part is None:
            part = self.partials[(M, N)] = torch.empty(M, N, dtype=torch.bfloat16, device=self.device)
        ops.gemm(x, w, b_t=w_t, out=part)
        work = dist.reduce_scatter_tensor(out, part, group=self.group, async_op=True)
        return lambda: self.wait(work)

    def _reduce_scatter(self, part: torch.Tensor, out, residual) -> torch.Tensor:
        M, N = part.shape
        if not self.sp:  # all-reduce: every rank keeps every row
            self.wait(dist.all_reduce(part, group=self.group, async_op=True))
            y = torch.empty(M, N, dtype=torch.bfloat16, device=self.device) if out is None else out
            y.copy_(part)
            if residual is not None:
                y.add_(residual)
            return y
        y = torch.empty(M // self.world, N, dtype=torch.bfloat16, device=self.device) if out is None else out
        self.wait(dist.reduce_scatter_tensor(y, part, group=self.group, async_op=True))
        if residual is not None:
            y.add_(residual)
        return y

    def close(self) -> None:
        pass


class FusedTP:
    """``TensorParallelComm`` (symmetric heap of this TP group) behind the stage interface."""

    def __init__(self, comm, sp: bool = True):
        self.comm = comm
        self.rank, self.world = comm.rank, comm.world
        self.sp = sp

    def chunk(self, M: int, K: int) -> torch.Tensor:
        return self.comm.local_chunk(M, K) if self.sp else self.comm.gather_buffer(M, K)

    def ag_gemm(self, M: int, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False):
        K = w.shape[0] if w_t else w.shape[1]
        x = self.comm.gather_buffer(M, K)
        if not self.sp:
            self.comm.advance_gather()
            return ops.gemm(x, w, b_t=w_t, out=out), x
        return self.comm.all_gather_gemm(M, w, out=out, w_t=w_t), x

    def all_gather(self, M: int, K: int) -> torch.Tensor:
        if not self.sp:
            x = self.comm.gather_buffer(M, K)
            self.comm.advance_gather()
            return x
        return self.comm.all_gather(M, K)

    def fp8_local(self, M: int, K: int):
        return self.comm.fp8_local(M, K) if self.sp else self.comm.fp8_views(M, K)

    def all_gather_fp8(self, M: int, K: int):
        if not self.sp:
            out = self.comm.fp8_views(M, K)
            self.comm.advance_gather()
            return out
        return self.comm.all_gather_fp8(M, K)

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, w_t: bool = False,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        if not self.sp:
            N = w.shape[1] if w_t else w.shape[0]
            return self._all_reduce(x.shape[0], N, lambda mine, res: self.comm.gemm_reduce_scatter(
                x, w, out=mine, w_t=w_t, residual=res), out, residual)
        return self.comm.gemm_reduce_scatter(x, w, out=out, w_t=w_t, residual=residual)

    def gemm_rs_with(self, M: int, N: int, gemm, out: torch.Tensor | None = None,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
        if not self.sp:
            return self._all_reduce(M, N, lambda mine, res: self.comm.reduce_scatter_with(
                M, N, gemm, out=mine, residual=res), out, residual)
        return self.comm.reduce_scatter_with(M, N, gemm, out=out, residual=residual)

    def gemm_rs_async(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, w_t: bool = False):
        if not self.sp:
            self.gemm_rs(x, w, out=out, w_t=w_t)
            return _done
        return self.comm.gemm_reduce_scatter_begin(x, w, out, w_t=w_t)

    def _all_reduce(self, M: int, N: int, reduce_scatter, out, residual) -> torch.Tensor:
        """GEMM -> all-reduce as GEMM -> reduce-scatter (this rank's reduced rows, plus the
        replicated residual's same rows, land in its gather chunk) and a peer all-gather."""
        rows = M // self.world
        mine = self.comm.local_chunk(M, N)
        res = None if residual is None else residual[self.rank * rows:(self.rank + 1) * rows]
        reduce_scatter(mine, res)
        full = self.comm.all_gather(M, N)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=full.device) if out is None else out
        y.copy_(full)
        return y

    def check(self) -> None:
        self.comm.heap.check()

    def close(self) -> None:
        self.comm.close()
