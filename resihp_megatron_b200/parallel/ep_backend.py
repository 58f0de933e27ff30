"""Expert-parallel MoE transport with library collectives, behind the peer-memory layer's interface.

``CollectiveEP`` runs the same phases as ``parallel.moe_ep.ExpertParallelMoE`` -- route,
exchange counts, dispatch, experts, combine, and their gradients -- with ``all_to_all_single``
(NCCL on GPUs, gloo on CPU), the reference's transport (``resihp/runtime/moe.py:149-265``).  It is
the baseline the peer-memory kernels are measured against and the transport of CPU tests.
Routing matches the kernels: fp32 logits of the bf16 input, experts selected on logits + bias,
softmax gates over the selected logits; receive rows at a holder are expert-major, then source
rank, then the (token, slot) order of the source -- the layout ``receive_layout`` defines.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .moe_ep import replica_cycles, replica_layout, split_count


class CollectiveEP:
    def __init__(self, rank: int, world: int, group, device, *, hidden: int, num_experts: int, top_k: int,
                 holder: list, waiter=None, speeds: dict[int, float] | None = None):
        self.rank, self.world, self.group = rank, world, group
        self.H, self.E, self.k = hidden, num_experts, top_k
        self.holders = [list(h) if isinstance(h, (list, tuple)) else [int(h)] for h in holder]
        self.cycles = replica_cycles(self.holders, speeds)
        self.local = [e for e in range(num_experts) if rank in self.holders[e]]
        self.device = torch.device(device)
        L = max(len(c) for c in self.cycles)
        self._cycle_t = torch.tensor([c + [c[0]] * (L - len(c)) for c in self.cycles], dtype=torch.int64,
                                     device=self.device)
        self._period_t = torch.tensor([len(c) for c in self.cycles], dtype=torch.int64, device=self.device)
        self.wait = waiter or (lambda w: w.wait())
        self.saved: dict = {}

    def take_state(self) -> dict:
        st, self.saved = self.saved, {}
        return st

    def put_state(self, state: dict) -> None:
        self.saved = state

    def _a2a(self, out, inp, out_splits, in_splits) -> None:
        if self.world == 1:
            out.copy_(inp)
            return
        self.wait(dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=True))

    # ------------------------------------------------------------------ forward
    def route(self, x: torch.Tensor, router_w: torch.Tensor, bias: torch.Tensor | None = None) -> None:
        logits = x.float() @ router_w.float().t()
        sel = logits if bias is None else logits + bias.float()
        topi = sel.topk(self.k, dim=-1).indices
        gates = torch.softmax(logits.gather(-1, topi), dim=-1)
        flat = topi.reshape(-1)
        n = flat.numel()
        idx = torch.arange(n, device=flat.device)
        counts = torch.bincount(flat, minlength=self.E).to(torch.int64)
        # position of every (token, slot) pair among this rank's pairs of its expert (token-major)
        by_expert = torch.argsort(flat * (n + 1) + idx)
        first = torch.cumsum(counts, 0) - counts
        pos = torch.empty_like(flat)
        pos[by_expert] = idx - first[flat[by_expert]]
        holder = self._cycle_t[flat, pos % self._period_t[flat]]
        # send order: by holder, then expert, then position
        order = torch.argsort((holder * self.E + flat) * (n + 1) + idx)
        self.saved = {"x": x, "topi": topi, "gates": gates, "T": x.shape[0], "counts": counts, "order": order}

    def exchange_counts(self) -> None:
        c = self.saved["counts"]
        table = torch.empty(self.world, self.E, dtype=torch.int64, device=c.device)
        if self.world == 1:
            table[0].copy_(c)
        else:
            self.wait(dist.all_gather_into_tensor(table.view(-1), c, group=self.group, async_op=True))
        self._layout(table.cpu())

    def set_counts_table(self, table: torch.Tensor) -> None:
        self._layout(table.cpu())

    def _layout(self, table: torch.Tensor) -> None:
        s = self.saved
        tab = table.tolist()
        s["table"] = table
        _, ranges = replica_layout(tab, self.cycles, self.rank, self.world)
        s["local_ranges"] = ranges
        s["recv_rows"] = sum(n for _, n in ranges)
        me, W, E = self.rank, self.world, self.E

        def cnt(src: int, e: int, h: int) -> int:
            return split_count(tab[src][e], self.cycles[e], h)

        # what this rank sends to holder h: its pairs dealt to h, expert order, position order
        s["send_splits"] = [sum(cnt(me, e, h) for e in range(E)) for h in range(W)]
        # what this rank receives from source r: r's pairs of this rank's experts, expert order
        s["recv_splits"] = [sum(cnt(r, e, me) for e in self.local) for r in range(W)]
        # receive order (source-major, expert) -> expert-major rows of the layout
        perm = []
        starts = {e: lo for e, (lo, _) in zip(self.local, ranges)}
        for r in range(W):
            for e in self.local:
                base = starts[e] + sum(cnt(q, e, me) for q in range(r))
                perm.extend(range(base, base + cnt(r, e, me)))
        s["perm"] = torch.tensor(perm, dtype=torch.int64, device=self.device)

    def dispatch(self) -> None:
        s = self.saved
        send = s["x"][s["order"] // self.k]  # the token of every pair, in send order
        recv = torch.empty(s["recv_rows"], self.H, dtype=send.dtype, device=self.device)
        tmp = torch.empty_like(recv)
        self._a2a(tmp, send, s["recv_splits"], s["send_splits"])
        recv[s["perm"]] = tmp
        s["recv"] = recv

    def experts_forward(self, weights, keep_input: bool = True) -> None:
        s = self.saved
        y = torch.empty_like(s["recv"])
        s["expert_cache"] = {}
        clock = getattr(self, "clock", None)
        if clock is not None:
            clock.begin(s["recv_rows"])
        for e, (lo, n) in zip(self.local, s["local_ranges"]):
            if n == 0:
                continue
            xin = s["recv"][lo:lo + n]
            w13, w2 = weights[e]
            gu = ops.gemm(xin, w13)
            a = ops.swiglu_fwd(gu)
            ops.gemm(a, w2, out=y[lo:lo + n])
            s["expert_cache"][e] = (gu, a, xin)
        if clock is not None:
            clock.end()
        s["y"] = y

    def combine(self, residual: torch.Tensor) -> torch.Tensor:
        s = self.saved
        back = torch.empty(s["order"].numel(), self.H, dtype=residual.dtype, device=self.device)
        self._a2a(back, s["y"][s["perm"]], s["send_splits"], s["recv_splits"])
        ycache = torch.empty_like(back)
        ycache[s["order"]] = back  # (token, slot) order
        s["ycache"] = ycache
        g = s["gates"].reshape(-1, 1)
        contrib = (ycache.float() * g).view(s["T"], self.k, self.H).sum(1)
        return (residual.float() + contrib).to(residual.dtype)

    def finish_forward(self) -> None:
        pass

    # ------------------------------------------------------------------ backward
    def grad_push(self, dout: torch.Tensor) -> None:
        s = self.saved
        rep = dout.float().repeat_interleave(self.k, 0)  # (token, slot) order
        g = s["gates"].reshape(-1, 1)
        s["dgate"] = (rep * s["ycache"].float()).sum(-1).view(s["T"], self.k)
        dy = (rep * g).to(dout.dtype)[s["order"]]
        tmp = torch.empty(s["recv_rows"], self.H, dtype=dout.dtype, device=self.device)
        self._a2a(tmp, dy, s["recv_splits"], s["send_splits"])
        dyrecv = torch.empty_like(tmp)
        dyrecv[s["perm"]] = tmp
        s["dyrecv"], s["dout"] = dyrecv, dout

    def experts_backward(self, weights, grads) -> None:
        s = self.saved
        dx = torch.zeros_like(s["dyrecv"])
        clock = getattr(self, "clock", None)
        if clock is not None:
            clock.begin(s["recv_rows"])
        for e, (lo, n) in zip(self.local, s["local_ranges"]):
            if n == 0:
                continue
            w13, w2 = weights[e]
            gu, a, xin = s["expert_cache"][e]
            dy = s["dyrecv"][lo:lo + n]
            da = ops.gemm(dy, w2, b_t=True)
            ops.gemm(dy, a, a_t=True, b_t=True, out=grads[e][1], accumulate=True)
            dgu = ops.swiglu_bwd(gu, da)
            ops.gemm(dgu, xin, a_t=True, b_t=True, out=grads[e][0], accumulate=True)
            ops.gemm(dgu, w13, b_t=True, out=dx[lo:lo + n])
        if clock is not None:
            clock.end()
        s["dxrecv"] = dx

    def grad_pull(self, router_w: torch.Tensor, router_grad: torch.Tensor, residual: bool = True,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        s = self.saved
        back = torch.empty(s["order"].numel(), self.H, dtype=s["dxrecv"].dtype, device=self.device)
        self._a2a(back, s["dxrecv"][s["perm"]], s["send_splits"], s["recv_splits"])
        pairs = torch.empty_like(back)
        pairs[s["order"]] = back
        dx = pairs.float().view(s["T"], self.k, self.H).sum(1)
        if residual:
            dx = dx + s["dout"].float()
        gates, dgate = s["gates"], s["dgate"]
        dsel = gates * (dgate - (gates * dgate).sum(-1, keepdim=True))
        dlogits = torch.zeros(s["T"], self.E, dtype=torch.float32, device=self.device)
        dlogits.scatter_(1, s["topi"], dsel)
        router_grad.add_(dlogits.t() @ s["x"].float())
        dx = dx + dlogits @ router_w.float()
        out = torch.empty(s["T"], self.H, dtype=s["dout"].dtype, device=self.device) if out is None else out
        out.copy_(dx)
        return out

    def close(self) -> None:
        pass
