"""GPU training engine for Mixtral-style MoE models: data parallel dense weights, expert parallel
experts over the same ranks (benchmark config 3: EP8 x DP8, TP1).

``GPUMoETrainer.train_step()`` runs one optimizer step of the global batch: rank ``r`` takes the
micro-batches ``[r * n, (r + 1) * n)`` of the step (synthetic tokens from ``TokenSource``, copied
from pinned host memory), runs every micro-batch forward and backward with the expert transport
(``ep_impl="peer"``: peer-memory kernels over NVLink; ``"collective"``: ``all_to_all``), reduces
the dense gradients data parallel (``dp_impl="fused"``: the fused peer-memory reduction + Adam +
gather; ``"collective"``: NCCL) and applies Adam to its dense shard and to its own experts (one
holder per expert: no expert reduction).  Returns the global mean token loss.
(Reference: the EP runtime, ``resihp/runtime/moe.py:149-269``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.config import GPTConfig


class ExpertSync:
    """Gradient reduction over the replicas of every replicated expert (one all-reduce per
    distinct holder set, experts in order) and Adam on this rank's expert copies (their optimizer
    state is replicated with them)."""

    def __init__(self, holders: list[list[int]], rank: int, device, waiter=None):
        self.holders = holders
        self.rank = rank
        self.device = torch.device(device)
        self.wait = waiter or (lambda w: w.wait())
        sets: dict[tuple[int, ...], list[int]] = {}
        for e, hs in enumerate(holders):
            sets.setdefault(tuple(sorted(hs)), []).append(e)
        self.groups = {}
        for hs in sorted(sets):  # every rank creates every group, in one order
            if len(hs) > 1:
                pg = dist.new_group(list(hs))
                if rank in hs:
                    self.groups[hs] = (pg, sets[hs])
        self.P = None

    def attach(self, P) -> None:
        self.P = P

    def reduce(self, layers: int) -> None:
        P = self.P
        for hs, (pg, experts) in sorted(self.groups.items()):
            views = [P.g(f"layers.{l}.experts.{e}.{w}") for l in range(layers) for e in experts for w in ("w13", "w2")]
            flat = torch.cat([v.reshape(-1) for v in views])
            self.wait(dist.all_reduce(flat, group=pg, async_op=True))
            off = 0
            for v in views:
                v.copy_(flat[off:off + v.numel()].view_as(v))
                off += v.numel()

    def apply(self, *, lr, betas, eps, weight_decay) -> None:
        from .. import ops

        P = self.P
        P.step += 1
        ops.adam_step(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.bf16, lr=lr, beta1=betas[0], beta2=betas[1],
                      eps=eps, weight_decay=weight_decay, step=P.step, zero_grad=True)


def _norm_holders(holder, world: int, E: int) -> list[list[int]]:
    if holder is None:
        return [[e * world // E] for e in range(E)]
    return [sorted(h) if isinstance(h, (list, tuple)) else [int(h)] for h in holder]


class GPUMoETrainer:
    def __init__(self, cfg: GPTConfig, *, global_batch: int, micro_batch: int = 1, seq_len: int | None = None,
                 ep_impl: str = "peer", dp_impl: str = "fused", seed: int = 0, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.0, device=None, data_seed: int = 1,
                 holder: list | None = None, speeds: dict[int, float] | None = None):
        """``holder[e]``: the rank of expert ``e`` or the list of its replicas' ranks (default:
        experts spread evenly); ``speeds``: relative speed per rank for dealing the tokens of a
        replicated expert."""
        from ..models.moe_model import MoEModel
        from ..runtime.gpu_executor import TokenSource
        from ..runtime.gpu_runtime import ParamSetSync

        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        if global_batch % (micro_batch * self.world):
            raise ValueError("the global batch must split into whole micro-batches on every rank")
        self.cfg = cfg
        self.S = seq_len or cfg.seq_len
        self.device = torch.device(device if device is not None else f"cuda:{torch.cuda.current_device()}")
        self.micro_batch = micro_batch
        self.n_local = global_batch // (micro_batch * self.world)
        self.global_batch = global_batch
        self.tokens_per_step = global_batch * self.S
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.ep_impl = ep_impl
        self.holders = _norm_holders(holder, self.world, cfg.num_experts)
        self.speeds = dict(speeds or {})
        self.abort = None
        if ep_impl == "peer":
            from ..parallel.symm import AbortWord

            self.abort = AbortWord()
        elif ep_impl != "collective":
            raise ValueError(ep_impl)
        self.ep = self._make_ep(self.holders, self.speeds)
        ranks = tuple(range(self.world))
        self.dense_sync = ParamSetSync(ranks, self.rank, None, dp_impl, self.device, abort=self.abort)
        self.model = MoEModel(cfg, self.device, ep=self.ep, holder=self.holders, rank=self.rank,
                              micro_batch=micro_batch, seq_len=self.S, seed=seed, dense_shard=self.dense_sync.shard,
                              dense_factories=self.dense_sync.factories)
        self.dense_sync.attach(self.model.dense)
        self.expert_sync = ExpertSync(self.holders, self.rank, self.device)
        self.expert_sync.attach(self.model.experts)
        self.tokens = TokenSource(cfg.vocab_size, micro_batch, self.S, seed=data_seed)
        self.iteration = 0
        self.h2d_bytes = 0
        self.layout = f"ep{self.world}dp{self.world}-{ep_impl}ep-{dp_impl}dp"
        self.last_reconfig: dict | None = None
        self.clock = None
        self.monitor = None
        self.failslow_events: list[dict] = []

    # ------------------------------------------------------------------ fail-slow detection
    def enable_failslow(self, *, slowdown: float = 1.0, model_ms_per_row: float | None = None,
                        **detector_kw) -> None:
        """Time this rank's expert compute every step and run the residual-BOCD monitor on every
        rank's times after each ``train_step``; a rank flagged slow triggers ``replace_experts``
        with its estimated speed.  ``slowdown`` > 1 emulates a slower GPU on this rank (host-side
        idling inside its expert regions; no GPU setting is touched); ``model_ms_per_row``
        replaces the measurement by a modelled time (CPU tests)."""
        from .moe_failslow import ExpertClock, ExpertSlowMonitor

        self.clock = ExpertClock(self.device, slowdown, model_ms_per_row, seed=self.rank)
        self.ep.clock = self.clock
        self.monitor = ExpertSlowMonitor(self.world, **detector_kw)

    def set_slowdown(self, factor: float) -> None:
        if self.clock is not None:
            self.clock.slowdown = float(factor)

    def _observe_failslow(self) -> dict | None:
        ms, rows = self.clock.collect()
        mine = torch.tensor([ms, float(rows)], dtype=torch.float64, device=self.device)
        allv = torch.empty(self.world * 2, dtype=torch.float64, device=self.device)
        if self.world > 1:
            dist.all_gather_into_tensor(allv, mine)
        else:
            allv.copy_(mine)
        v = allv.view(self.world, 2).tolist()
        slow = self.monitor.observe(self.iteration - 1, [a for a, _ in v], [int(b) for _, b in v])
        if not slow:
            return None
        speeds = {r: max(0.05, min(1.0, p)) for r, p in slow.items()}
        info = self.replace_experts(speeds)
        self.monitor.reset()
        event = {"iteration": self.iteration - 1, "speeds": speeds, "holders": info["holders"]}
        self.failslow_events.append(event)
        return event

    def _make_ep(self, holders, speeds):
        cfg, T = self.cfg, self.micro_batch * self.S
        if self.ep_impl == "peer":
            from ..parallel.moe_ep import ExpertParallelMoE
            from ..parallel.symm import exchange_via_group

            return ExpertParallelMoE(self.rank, self.world, exchange_via_group(None), self.device, hidden=cfg.hidden,
                                     num_experts=cfg.num_experts, top_k=cfg.top_k, max_tokens=T, holder=holders,
                                     abort=self.abort, speeds=speeds)
        from ..parallel.ep_backend import CollectiveEP

        return CollectiveEP(self.rank, self.world, None, self.device, hidden=cfg.hidden, num_experts=cfg.num_experts,
                            top_k=cfg.top_k, holder=holders, speeds=speeds)

    def step_device(self) -> torch.Tensor:
        """One step; the global mean loss as a 0-d device tensor (no host synchronisation)."""
        m = self.model
        m.loss_acc.zero_()
        scale = 1.0 / self.tokens_per_step
        self.h2d_bytes = 0
        for j in range(self.n_local):
            ids, labels = self.tokens.tokens(self.iteration, self.rank * self.n_local + j)
            self.h2d_bytes += ids.numel() * ids.element_size() + labels.numel() * labels.element_size()
            m.forward_backward(ids.to(self.device, non_blocking=True), labels.to(self.device, non_blocking=True),
                               scale)
        kw = dict(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.wd)
        self.dense_sync.step(**kw)
        self.expert_sync.reduce(self.cfg.layers)
        self.expert_sync.apply(**kw)
        loss = m.loss_acc.clone()
        if self.world > 1:
            dist.all_reduce(loss)
        self.iteration += 1
        return loss / self.tokens_per_step

    @property
    def h2d_bytes_last_step(self) -> int:
        return self.h2d_bytes

    def train_step(self) -> float:
        """One step through the public path; with fail-slow detection enabled, the step's expert
        times are then exchanged and a flagged rank's experts re-placed before the next step."""
        value = float(self.step_device().item())
        self.check()
        if self.monitor is not None:
            self._observe_failslow()
        return value

    # ------------------------------------------------------------------ expert re-placement
    def expert_specs(self) -> dict:
        from ..state.layer_registry import TensorSpec

        c = self.cfg
        out = {}
        for l in range(c.layers):
            for e in range(c.num_experts):
                for w, shape in (("w13", (2 * c.ffn, c.hidden)), ("w2", (c.hidden, c.ffn))):
                    k = f"layers.{l}.experts.{e}.{w}"
                    out[k] = TensorSpec(k, shape, None)
        return out

    def replace_experts(self, speeds: dict[int, float], loads: list[float] | None = None,
                        holder: list | None = None) -> dict:
        """Re-place the experts between steps for the relative ``speeds`` of the ranks (a
        fail-slow GPU): the placement planner (``plan.expert_placement``) may replicate a slow
        rank's experts on faster ranks and deal their tokens by speed; the expert weights and
        Adam moments move slice by slice (peer to peer over NVLink on GPUs, else send/receive),
        dense weights stay.  Every rank calls it; ``holder`` overrides the planner.  Returns the
        new placement and phase timings.  (Reference: resilient expert placement,
        ``resihp/plan/expert_placement.py``, and the EP runtime's state migration.)"""
        import time

        from ..plan.expert_placement import ExpertPlacement, plan_expert_placement
        from ..state.transfer_engine import execute_transfers
        from ..state.transfer_plan import plan_transfers

        marks = [("start", time.perf_counter())]

        def mark(name):
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            marks.append((name, time.perf_counter()))

        W, E = self.world, self.cfg.num_experts
        ids = [str(r) for r in range(W)]
        old = ExpertPlacement(E, (tuple(ids),), {ids[r]: tuple(e for e in range(E) if r in self.holders[e])
                                                 for r in range(W)})
        if holder is None:
            new = plan_expert_placement([ids], E, speeds={ids[r]: v for r, v in speeds.items()}, loads=loads,
                                        prev=old, slots_per_device=-(-E // W) + 1)
            new_holders = [sorted(int(d) for d in new.holders(e)) for e in range(E)]
        else:
            new_holders = _norm_holders(holder, W, E)
        mark("plan")
        specs = self.expert_specs()

        def hold(holders):
            return {k: [(ids[r], (0, 1)) for r in holders[int(k.split(".")[3])]] for k in specs}

        old_h, new_h = hold(self.holders), hold(new_holders)
        tplan = plan_transfers(old_h, new_h, valid_sources=set(ids), node_of={d: "n0" for d in ids})
        P = self.model.experts
        kinds = ("param", "exp_avg", "exp_avg_sq")
        old_state = {k: {} for k in kinds}
        for name in P.order:
            for kind, buf in zip(kinds, (P.master, P.exp_avg, P.exp_avg_sq)):
                o, n = P.offsets[name], P.specs[name].numel
                old_state[kind][name] = buf[o:o + n].view(P.specs[name].shape)
        me = ids[self.rank]
        new_local = [e for e in range(E) if self.rank in new_holders[e]]
        wanted = [k for k in specs if int(k.split(".")[3]) in new_local]
        if self.device.type == "cuda":
            from ..parallel.migration import migrate_p2p
            from ..parallel.symm import exchange_via_group

            new_state = {kd: {k: torch.empty(specs[k].global_shape, dtype=torch.float32, device=self.device)
                              for k in wanted} for kd in kinds}
            migrate_p2p(tplan, me, ids, specs=specs, old_h=old_h, new_h=new_h, old_state=old_state,
                        new_state=new_state, kinds=kinds, device=self.device, exchange=exchange_via_group(None))
        else:
            new_state = execute_transfers(tplan, me, _World(ids), _NoWait(),
                                          specs=specs, old_layout={k: (0, 1) for k in old_state["param"]},
                                          old_state=old_state, new_layout={k: (0, 1) for k in wanted}, kinds=kinds,
                                          dtype=torch.float32, device=str(self.device))
        mark("migrate")
        step = P.step
        self.ep.close()
        self.holders, self.speeds = new_holders, dict(speeds)
        self.ep = self._make_ep(self.holders, self.speeds)
        if self.clock is not None:
            self.ep.clock = self.clock
        self.model.rebuild_experts(self.holders, self.rank, self.ep)
        Q = self.model.experts
        for name in Q.order:
            o, n = Q.offsets[name], Q.specs[name].numel
            for kind, buf in zip(kinds, (Q.master, Q.exp_avg, Q.exp_avg_sq)):
                buf[o:o + n].copy_(new_state[kind][name].reshape(-1))
            Q.w(name).copy_(new_state["param"][name])
        Q.step = step
        self.expert_sync = ExpertSync(self.holders, self.rank, self.device)
        self.expert_sync.attach(Q)
        mark("commit")
        self.last_reconfig = {name: round(t - marks[i][1], 4) for i, (name, t) in enumerate(marks[1:])}
        self.last_reconfig.update(holders=self.holders, transfers=len(tplan.transfers))
        return self.last_reconfig

    def check(self) -> None:
        self.dense_sync.check()
        heap = getattr(self.ep, "heap", None)
        if heap is not None:
            heap.check()

    def close(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.dense_sync.close()
        self.ep.close()
        if self.abort is not None:
            self.abort.close()
            self.abort = None


class _World:
    """The default group as the transfer engine's communicator view (device ids are ranks)."""

    def __init__(self, ids: list[str]):
        self.ids = ids

    def rank_of(self, device: str) -> int:
        return self.ids.index(device)


class _NoWait:
    """Waits on a work object directly (the transfer engine's ``guarded_wait`` without a control plane)."""

    @staticmethod
    def guarded_wait(work, timeout=None, what=""):
        work.wait()
