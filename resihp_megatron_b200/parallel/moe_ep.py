"""Expert-parallel MoE layer on GPUs: routing, dispatch and combine over NVLink peer memory.

One layer ``y = x + sum_k g_k(x) E_{e_k}(x)`` (top-k routing, softmax over the selected logits, a
non-trainable bias that only selects, SwiGLU experts ``w2 (silu(x w1^T) * (x w3^T))`` with
``w13 = [w1; w3]``).  Expert ``e`` lives on rank ``holder[e]``.  Per step:

1. ``moe_route`` (router kernel) and ``moe_positions`` (fixed-order ranks of each (token, slot)
   within its expert) on every rank; the per-expert counts go to the symmetric heap.
2. Bounded barrier, every rank pulls all count vectors (one slice-copy launch), and the host derives
   each expert's receive rows: expert-major, then source rank, then position -- a layout that does
   not depend on timing, so expert weight gradients are fixed-order sums.
3. ``moe_dispatch``: every (token, slot) row is stored straight into its holder's receive buffer.
4. Barrier; each holder runs its local experts' GEMMs on contiguous row ranges (tcgen05 kernels).
5. Barrier; ``moe_combine`` pulls the expert outputs back and adds them with the gates.
Backward mirrors it (``moe_grad_push`` / expert backward / ``moe_grad_pull``).

Replaces the reference's EP runtime transport (``resihp/runtime/moe.py:149-265``: counts
all-to-all, autograd ``all_to_all_single``, ``index_add``).  Placement changes (expert
re-placement after a fail-slow) only change ``holder``; expert state moves with ``symm_copy``.
"""

from __future__ import annotations

import torch

from .. import ops
from ..ops._build import ext
from .symm import AbortWord, SymmetricHeap


PERIOD_MAX = 64  # longest replica cycle the dispatch kernel takes
HOLDERS_MAX = 16


def replica_cycles(holders: list[list[int]], speeds: dict[int, float] | None = None) -> list[list[int]]:
    """Per expert, the holder of every slot of its dealing cycle: the (token, slot) pair at
    position ``p`` of expert ``e`` on any source goes to ``cycle[e][p % len(cycle[e])]`` -- one
    period of the speed-weighted smooth round robin the CPU runtime uses
    (``plan.expert_placement.smooth_weighted_round_robin``, integer weights ``10 * speed``)."""
    from ..plan.expert_placement import smooth_weighted_round_robin

    speeds = speeds or {}
    out = []
    for hs in holders:
        hs = list(hs)
        if len(hs) == 1:
            out.append(hs)
            continue
        period = sum(max(1, round(10 * speeds.get(h, 1.0))) for h in hs)
        if period > PERIOD_MAX:
            raise ValueError(f"replica cycle of {period} slots exceeds {PERIOD_MAX}")
        out.append(smooth_weighted_round_robin(hs, speeds, period))
    return out


def split_count(count: int, cycle: list[int], holder: int) -> int:
    """Pairs among the first ``count`` positions of an expert that its cycle deals to ``holder``."""
    full, rem = divmod(int(count), len(cycle))
    return full * cycle.count(holder) + cycle[:rem].count(holder)


def replica_layout(table, cycles: list[list[int]], me: int, world: int):
    """Receive rows of a step from the count table ``table[source][expert]``: at every holder its
    experts in expert order, each expert's rows ordered by source rank, then by position.  Returns
    ``rowbase[e][h]`` -- the first row, at holder ``h``, of this source's (``me``'s) pairs of
    expert ``e`` -- and, for ``me`` as a holder, the ``(first row, rows)`` range of each expert it
    holds (expert order)."""
    E = len(cycles)
    cnt = [[[split_count(table[s][e], cycles[e], h) for h in range(world)] for e in range(E)] for s in range(world)]
    start: dict[tuple[int, int], int] = {}
    for h in range(world):
        off = 0
        for e in range(E):
            if h in cycles[e]:
                start[(e, h)] = off
                off += sum(cnt[s][e][h] for s in range(world))
    rowbase = [[0] * world for _ in range(E)]
    for (e, h), lo in start.items():
        rowbase[e][h] = lo + sum(cnt[s][e][h] for s in range(me))
    ranges = [(start[(e, me)], sum(cnt[s][e][me] for s in range(world))) for e in range(E) if me in cycles[e]]
    return rowbase, ranges


def receive_capacity(holders: list[list[int]], world: int, max_tokens: int) -> int:
    """Rows of every rank's receive segments.  The heap is symmetric: every rank must lay out the
    same segment sizes, or a peer's segment offsets differ from this rank's and stores meant for
    a peer's buffer land outside it.  So the size is the same on every rank -- that of the rank
    holding the most experts (a speed-weighted placement gives ranks different expert counts);
    each source rank sends at most ``max_tokens`` rows per expert."""
    most_local = max(sum(1 for h in holders if r in h) for r in range(world))
    return max_tokens * world * max(1, most_local)


def receive_layout(table, holder: list[int], me: int, world: int) -> tuple[list[int], list[tuple[int, int]]]:
    """``replica_layout`` for one holder per expert: ``rowbase[e]`` at ``holder[e]``."""
    rowbase, ranges = replica_layout(table, [[h] for h in holder], me, world)
    return [rowbase[e][holder[e]] for e in range(len(holder))], ranges


class ExpertParallelMoE:
    def __init__(self, rank: int, world: int, exchange, device, *, hidden: int, num_experts: int, top_k: int,
                 max_tokens: int, holder: list, abort: AbortWord | None = None, budget_s: float = 30.0,
                 speeds: dict[int, float] | None = None, _heap: SymmetricHeap | None = None):
        """``holder[e]``: the rank of expert ``e``, or the list of its replicas' ranks (the pairs
        routed to a replicated expert are dealt to its replicas by ``replica_cycles`` with
        ``speeds``)."""
        self.rank, self.world = rank, world
        self.H, self.E, self.k = hidden, num_experts, top_k
        self.holders = [list(h) if isinstance(h, (list, tuple)) else [int(h)] for h in holder]
        self.cycles = replica_cycles(self.holders, speeds)
        self.local = [e for e in range(num_experts) if rank in self.holders[e]]
        self.max_rows = receive_capacity(self.holders, world, max_tokens)
        self.device = torch.device(device)
        self.abort, self.budget = abort, budget_s
        segs = {"counts": (world * 16, torch.int32),
                "recv": (self.max_rows * hidden, torch.bfloat16), "y": (self.max_rows * hidden, torch.bfloat16),
                "dyrecv": (self.max_rows * hidden, torch.bfloat16), "dxrecv": (self.max_rows * hidden, torch.bfloat16)}
        self.heap = _heap or SymmetricHeap(segs, rank, world, exchange, device, abort)
        self.emulated = _heap is not None
        routes = torch.zeros(num_experts, 2 * PERIOD_MAX + HOLDERS_MAX, dtype=torch.int32)
        for e, cyc in enumerate(self.cycles):
            for j, h in enumerate(cyc):
                routes[e, j] = h
                routes[e, PERIOD_MAX + j] = cyc[:j].count(h)
            for h in set(cyc):
                routes[e, 2 * PERIOD_MAX + h] = cyc.count(h)
        self.period_t = torch.tensor([len(c) for c in self.cycles], dtype=torch.int32, device=self.device)
        self.routes_t = routes.to(self.device)
        self.saved: dict = {}

    @classmethod
    def emulated_group(cls, world: int, device, **kw) -> list["ExpertParallelMoE"]:
        """``world`` ranks in one process on one GPU (tests); call each phase on every rank in turn."""
        E = kw["num_experts"]
        holders = [list(h) if isinstance(h, (list, tuple)) else [h] for h in kw["holder"]]
        rows = receive_capacity(holders, world, kw["max_tokens"])
        H = kw["hidden"]
        segs = {"counts": (world * 16, torch.int32), "recv": (rows * H, torch.bfloat16), "y": (rows * H, torch.bfloat16),
                "dyrecv": (rows * H, torch.bfloat16), "dxrecv": (rows * H, torch.bfloat16)}
        heaps = SymmetricHeap.emulated(segs, world, device)
        return [cls(r, world, None, device, _heap=heaps[r], **kw) for r in range(world)]

    def _barrier(self) -> None:
        if not self.emulated:
            self.heap.barrier(self.budget)

    def rows(self, name: str, n: int) -> torch.Tensor:
        return self.heap.tensor(name)[: n * self.H].view(n, self.H)

    # ------------------------------------------------------------------ phase 1: route
    def route(self, x: torch.Tensor, router_w: torch.Tensor, bias: torch.Tensor | None = None) -> None:
        T = x.shape[0]
        logits = torch.empty(T, self.E, dtype=torch.float32, device=x.device)
        topi = torch.empty(T, self.k, dtype=torch.int32, device=x.device)
        gates = torch.empty(T, self.k, dtype=torch.float32, device=x.device)
        ext().moe_route(x, router_w, bias, self.k, logits, topi, gates)
        pos = torch.empty_like(topi)
        counts = self.heap.tensor("counts")[self.rank * 16:(self.rank + 1) * 16]
        counts.zero_()
        ext().moe_positions(topi, self.E, pos, counts)
        ops.count(2)
        self.saved = {"x": x, "logits": logits, "topi": topi, "gates": gates, "pos": pos, "T": T}

    # ------------------------------------------------------------------ phase 2: counts
    def exchange_counts(self) -> None:
        """Pull every rank's count vector into this rank's table; derive receive rows."""
        self._barrier()
        base = self.heap.peer_ptrs("counts")
        me = self.rank
        triples = []
        for r in range(self.world):
            if r != me:
                triples += [base[r] + r * 64, base[me] + r * 64, 64]
        if triples:
            ext().symm_copy(triples, self.device.index if self.device.index is not None else 0)
        table = self.heap.tensor("counts").view(self.world, 16)[:, : self.E].to("cpu", torch.int64)
        self._layout(table)

    def set_counts_table(self, table: torch.Tensor) -> None:
        """Emulated groups: the full [world, E] count table (every rank's counts)."""
        self._layout(table.to("cpu", torch.int64))

    def _layout(self, table: torch.Tensor) -> None:
        rowbase, ranges = replica_layout(table.tolist(), self.cycles, self.rank, self.world)
        rb = torch.zeros(self.E, HOLDERS_MAX, dtype=torch.int64)
        rb[:, : self.world] = torch.tensor(rowbase, dtype=torch.int64)
        self.saved["rowbase"] = rb.to(self.device)
        self.saved["local_ranges"] = ranges
        self.saved["recv_rows"] = sum(n for _, n in ranges)

    # ------------------------------------------------------------------ phase 3: dispatch
    def dispatch(self) -> None:
        s = self.saved
        route_row = torch.empty(s["T"] * self.k, dtype=torch.int64, device=self.device)
        ext().moe_dispatch(s["x"], s["topi"], s["pos"], self.k, self.rank, self.period_t, self.routes_t, s["rowbase"],
                           self.heap.peer_ptrs("recv"), route_row)
        ops.count(1)
        s["route_row"] = route_row
        self._barrier()

    # ------------------------------------------------------------------ phase 4: experts
    def experts_forward(self, weights: dict[int, tuple[torch.Tensor, torch.Tensor]], keep_input: bool = False) -> None:
        """``weights[e] = (w13 [2F, H], w2 [H, F])`` for this rank's experts.  ``keep_input``
        copies the received rows out of the shared receive buffer, so the backward still has
        them after later layers reused the buffer (a multi-layer model keeps one ``saved`` state
        per layer: ``take_state`` / ``put_state``)."""
        s = self.saved
        s["expert_cache"] = {}
        clock = getattr(self, "clock", None)
        if clock is not None:
            clock.begin(s["recv_rows"])
        for e, (lo, n) in zip(self.local, s["local_ranges"]):
            if n == 0:
                continue
            xin = self.rows("recv", lo + n)[lo:]
            if keep_input:
                xin = xin.clone()
            w13, w2 = weights[e]
            gu = ops.gemm(xin, w13)
            a = ops.swiglu_fwd(gu)
            ops.gemm(a, w2, out=self.rows("y", lo + n)[lo:])
            s["expert_cache"][e] = (gu, a, xin if keep_input else None)
        if clock is not None:
            clock.end()  # before the barrier: a slow peer does not stretch this rank's time
        self._barrier()

    def take_state(self) -> dict:
        """Detach the routing / activation state of the layer just run (for its backward)."""
        st, self.saved = self.saved, {}
        return st

    def put_state(self, state: dict) -> None:
        self.saved = state

    # ------------------------------------------------------------------ phase 5: combine
    def combine(self, residual: torch.Tensor) -> torch.Tensor:
        s = self.saved
        out = torch.empty_like(residual)
        ycache = torch.empty(s["T"] * self.k, self.H, dtype=torch.bfloat16, device=self.device)
        ext().moe_combine(residual, s["gates"], s["route_row"], self.k, self.heap.peer_ptrs("y"), out, ycache)
        ops.count(1)
        s["ycache"] = ycache
        return out

    def finish_forward(self) -> None:
        self._barrier()  # holders may reuse their buffers

    # ------------------------------------------------------------------ backward
    def grad_push(self, dout: torch.Tensor) -> None:
        s = self.saved
        dgate = torch.empty(s["T"] * self.k, dtype=torch.float32, device=self.device)
        ext().moe_grad_push(dout, s["gates"], s["ycache"], s["route_row"], self.k, self.heap.peer_ptrs("dyrecv"),
                            dgate)
        ops.count(1)
        s["dgate"], s["dout"] = dgate, dout
        self._barrier()

    def experts_backward(self, weights, grads) -> None:
        """``grads[e] = (dw13 fp32, dw2 fp32)`` accumulated (fixed row order)."""
        s = self.saved
        clock = getattr(self, "clock", None)
        if clock is not None:
            clock.begin(s["recv_rows"])
        for e, (lo, n) in zip(self.local, s["local_ranges"]):
            if n == 0:
                continue
            w13, w2 = weights[e]
            gu, a, kept = s["expert_cache"][e]
            dy = self.rows("dyrecv", lo + n)[lo:]
            xin = kept if kept is not None else self.rows("recv", lo + n)[lo:]
            da = ops.gemm(dy, w2, b_t=True)
            ops.gemm(dy, a, a_t=True, b_t=True, out=grads[e][1], accumulate=True)
            dgu = ops.swiglu_bwd(gu, da)
            ops.gemm(dgu, xin, a_t=True, b_t=True, out=grads[e][0], accumulate=True)
            ops.gemm(dgu, w13, b_t=True, out=self.rows("dxrecv", lo + n)[lo:])
        if clock is not None:
            clock.end()
        self._barrier()

    def grad_pull(self, router_w: torch.Tensor, router_grad: torch.Tensor, residual: bool = True,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """Input gradient of the layer: expert paths + router path, plus the residual path when
        ``residual`` (the experts read the residual stream itself; False when they read a
        normalised copy, as in a transformer block); accumulates the router weight gradient
        (fp32) into ``router_grad``."""
        s = self.saved
        T = s["T"]
        dx = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device) if out is None else out
        dlogits = torch.empty(T, self.E, dtype=torch.float32, device=self.device)
        # dx = residual path + expert paths + router path (dl W_r), all in one pass per token
        ext().moe_grad_pull(s["dout"] if residual else None, s["gates"], s["dgate"], s["topi"], s["route_row"], self.k,
                            self.E, self.heap.peer_ptrs("dxrecv"), dx, dlogits, router_w.contiguous())
        # router weight gradient dl^T x: E <= 16 rows, too narrow for the tensor-core tiles
        ext().moe_router_wgrad(dlogits, s["x"].contiguous(), router_grad)
        ops.count(3)
        self._barrier()
        return dx

    def close(self) -> None:
        if not self.emulated or self.rank == 0:
            self.heap.close()
