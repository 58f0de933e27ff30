"""The float64 MoE block and a dropless expert-parallel runtime over arbitrary placements.

``y = x + sum_k g_k(x) * E_{e_k}(x)``: top-k routing whose softmax runs over the selected
logits; a non-trainable per-expert bias is added to the logits for *selection only*
(aux-loss-free balancing, moved by ``rate * sign(mean load - load)`` after every iteration).
Experts are two-layer GELU MLPs.  Parameters are a pure function of ``(seed, key)``, so every
placement trains the same model.

``EPRuntime`` replicates the router (data parallel over all ranks).  The (token, slot) pairs of
each expert are dealt to its replicas inside the EP group by speed-weighted smooth round robin;
a counts all-to-all precedes an autograd-aware all-to-all of the token rows, the local expert
copies run, a reverse all-to-all returns their outputs, and the outputs are combined with the
gate weights.  Each expert's gradient is summed over all its holders (``edp/`` groups that
follow from the placement).  Dropless routing and a per-token loss over the global token count
make any placement -- replicated experts or not, before or after a failure -- equal to the
single-process reference up to reduction order.  On GPUs the dispatch, expert GEMMs and combine
are the peer-memory kernels of ``parallel/moe_ep``.
Parity: ``resihp/runtime/moe.py:29-269`` (same model, routing, placement use and group names).
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..plan.expert_placement import ExpertPlacement, expert_dp_groups, smooth_weighted_round_robin
from ..state.layer_registry import FULL, Holdings, TensorSpec
from ..state.rng_data import generator
from ..utils.intervals import even_split

_EXPERT_MATS = ("fc1.weight", "fc2.weight")


@dataclass(frozen=True)
class MoEConfig:
    hidden: int = 8
    ffn: int = 12
    num_experts: int = 6
    top_k: int = 2
    tokens: int = 48
    seed: int = 4321
    dtype: torch.dtype = torch.float64
    bias_update_rate: float = 0.0


def _expert_key(e: int, mat: str) -> str:
    return f"experts.{e}.{mat}"


def moe_specs(cfg: MoEConfig) -> dict[str, TensorSpec]:
    """Registry specs: the router, the optional selection bias and every expert's two matrices."""
    shapes = {"fc1.weight": (cfg.ffn, cfg.hidden), "fc2.weight": (cfg.hidden, cfg.ffn)}
    specs = {"router.weight": TensorSpec("router.weight", (cfg.num_experts, cfg.hidden), None)}
    if cfg.bias_update_rate:
        specs["router.expert_bias"] = TensorSpec("router.expert_bias", (cfg.num_experts,), None, trainable=False)
    for e in range(cfg.num_experts):
        for mat in _EXPERT_MATS:
            key = _expert_key(e, mat)
            specs[key] = TensorSpec(key, shapes[mat], None)
    return specs


def expert_of(key: str) -> int | None:
    head, _, rest = key.partition(".")
    return int(rest.partition(".")[0]) if head == "experts" else None


def init_param(cfg: MoEConfig, spec: TensorSpec) -> torch.Tensor:
    if not spec.trainable:
        return torch.zeros(spec.global_shape, dtype=cfg.dtype)
    g = generator(cfg.seed, zlib.crc32(spec.key.encode()))
    fan_in = spec.global_shape[-1]
    return torch.randn(spec.global_shape, generator=g, dtype=cfg.dtype) / fan_in ** 0.5


def update_expert_bias(cfg: MoEConfig, bias: torch.Tensor, loads: torch.Tensor) -> None:
    """Aux-loss-free balancing: underloaded experts' bias rises, overloaded ones' falls."""
    with torch.no_grad():
        bias += cfg.bias_update_rate * (loads.mean() - loads).sign()


def batch(cfg: MoEConfig, iteration: int) -> tuple[torch.Tensor, torch.Tensor]:
    x = torch.randn(cfg.tokens, cfg.hidden, generator=generator(cfg.seed, iteration, 5), dtype=cfg.dtype)
    teacher = torch.randn(cfg.hidden, cfg.hidden, generator=generator(cfg.seed, 3), dtype=cfg.dtype)
    return x, torch.tanh(x @ teacher)


def route(cfg: MoEConfig, x: torch.Tensor, router: torch.Tensor, bias: torch.Tensor | None = None):
    """Top-k expert ids (chosen on logits + bias) and the softmax gates of the chosen logits."""
    logits = x @ router.t()
    chooser = logits if bias is None else logits + bias
    chosen = chooser.topk(cfg.top_k, dim=-1).indices
    return chosen, logits.gather(-1, chosen).softmax(dim=-1)


def expert_ffn(x: torch.Tensor, fc1: torch.Tensor, fc2: torch.Tensor) -> torch.Tensor:
    return F.linear(F.gelu(F.linear(x, fc1)), fc2)


def token_loss(out: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    return (out - y).pow(2).mean(dim=-1).sum()


def reference_forward(cfg: MoEConfig, params: dict[str, torch.Tensor], x: torch.Tensor) -> torch.Tensor:
    chosen, gates = route(cfg, x, params["router.weight"], params.get("router.expert_bias"))
    bias = params.get("router.expert_bias")
    if bias is not None:
        update_expert_bias(cfg, bias, torch.bincount(chosen.flatten(), minlength=cfg.num_experts).to(cfg.dtype))
    mixed = torch.zeros_like(x)
    for e in range(cfg.num_experts):
        tok, slot = torch.nonzero(chosen == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        y = expert_ffn(x[tok], params[_expert_key(e, "fc1.weight")], params[_expert_key(e, "fc2.weight")])
        mixed = mixed.index_add(0, tok, gates[tok, slot, None] * y)
    return x + mixed


def reference_train(cfg: MoEConfig, iterations: int, lr: float = 1e-2):
    """Single-process ground truth: losses per iteration and the final parameters and buffers."""
    from .optim import Adam

    specs = moe_specs(cfg)
    params = {k: torch.nn.Parameter(init_param(cfg, s)) for k, s in specs.items() if s.trainable}
    buffers = {k: init_param(cfg, s) for k, s in specs.items() if not s.trainable}
    opt = Adam(params, lr=lr)
    history = []
    for it in range(iterations):
        opt.zero_grad()
        x, y = batch(cfg, it)
        loss = token_loss(reference_forward(cfg, params | buffers, x), y)
        (loss / cfg.tokens).backward()
        opt.step()
        history.append(loss.item() / cfg.tokens)
    final = {k: v.detach().clone() for k, v in params.items()} | {k: v.clone() for k, v in buffers.items()}
    return history, final


def moe_holdings(placement: ExpertPlacement, specs: dict[str, TensorSpec]) -> Holdings:
    """Dense keys on every device, an expert's keys on its holders."""
    everyone = sorted(d for g in placement.groups for d in g)

    def holders(key: str) -> list[str]:
        e = expert_of(key)
        return everyone if e is None else placement.holders(e)

    return {key: [(d, FULL) for d in holders(key)] for key in specs}


def edp_group_name(holders: tuple[str, ...]) -> str:
    return "edp/" + ",".join(holders)


def moe_group_specs(placement: ExpertPlacement, world: list[str]):
    """``dp`` over everyone, ``ep/<i>`` per EP group, ``edp/<holders>`` per replicated expert set."""
    from ..comm.group_spec import GroupSpec

    rank_of = {d: r for r, d in enumerate(world)}

    def ranks(devices) -> tuple[int, ...]:
        return tuple(sorted(rank_of[d] for d in devices))

    specs = [GroupSpec("dp", tuple(range(len(world))), kind="dp")]
    specs += [GroupSpec(f"ep/{i}", ranks(g), kind="ep") for i, g in enumerate(placement.groups)]
    specs += [GroupSpec(edp_group_name(h), ranks(h), kind="edp") for h in expert_dp_groups(placement) if len(h) > 1]
    return specs


def _exchange(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group, wait) -> torch.Tensor:
    """``all_to_all_single`` (a plain copy without a group)."""
    if group is None:
        return out.copy_(inp)
    wait(dist.all_to_all_single(out, inp.contiguous(), out_splits, in_splits, group=group, async_op=True))
    return out


class _AllToAll(torch.autograd.Function):
    """All-to-all whose backward is the transposed all-to-all."""

    @staticmethod
    def forward(ctx, x, out_splits, in_splits, group, wait):
        ctx.meta = (out_splits, in_splits, group, wait)
        return _exchange(x.new_empty((sum(out_splits), *x.shape[1:])), x, out_splits, in_splits, group, wait)

    @staticmethod
    def backward(ctx, g):
        out_splits, in_splits, group, wait = ctx.meta
        back = _exchange(g.new_empty((sum(in_splits), *g.shape[1:])), g, in_splits, out_splits, group, wait)
        return back, None, None, None, None


class EPRuntime:
    """One MoE block on one device: the replicated router and the expert copies placed here."""

    def __init__(self, cfg: MoEConfig, placement: ExpertPlacement, me: str, world: list[str], comms, mgr,
                 params: dict[str, torch.Tensor], speeds: dict[str, float] | None = None, timeout: float = 60.0,
                 buffers: dict[str, torch.Tensor] | None = None):
        self.cfg, self.placement, self.me, self.world = cfg, placement, me, list(world)
        self.comms, self.mgr, self.timeout = comms, mgr, timeout
        self.speeds = speeds or {}
        self.params, self.buffers = params, buffers or {}
        self.gidx = placement.group_of(me)
        self.ep = sorted(placement.groups[self.gidx], key=self.world.index)
        self.local_experts = placement.slots[me]
        self.tokens_per_expert = None

    def wait(self, work) -> None:
        self.mgr.guarded_wait(work, timeout=self.timeout, what="moe")

    def token_range(self) -> tuple[int, int]:
        return even_split(self.cfg.tokens, len(self.world))[self.world.index(self.me)]

    def _destinations(self, chosen: torch.Tensor) -> torch.Tensor:
        """EP-group index of the holder each (token, slot) pair goes to (smooth weighted round
        robin over an expert's holders, pairs in token-major order)."""
        dest = torch.empty_like(chosen)
        where = {d: i for i, d in enumerate(self.ep)}
        for e in range(self.cfg.num_experts):
            tok, slot = torch.nonzero(chosen == e, as_tuple=True)
            if tok.numel():
                picks = smooth_weighted_round_robin(self.placement.group_holders(self.gidx, e), self.speeds, tok.numel())
                dest[tok, slot] = torch.tensor([where[p] for p in picks], dtype=dest.dtype)
        return dest

    def _pack(self, chosen: torch.Tensor, dest: torch.Tensor):
        """Send order (destination, expert, token, slot) and the ``[ep, experts]`` counts."""
        T, K = chosen.shape
        E = self.cfg.num_experts
        flat = torch.arange(T * K)
        key = (dest.flatten() * E + chosen.flatten()) * (T * K) + flat
        order = key.argsort()
        counts = torch.bincount(dest.flatten() * E + chosen.flatten(), minlength=len(self.ep) * E)
        return order // K, order % K, counts.view(len(self.ep), E)

    def _run_experts(self, recv: torch.Tensor, recv_counts: torch.Tensor) -> torch.Tensor:
        outputs, at = [], 0
        for src, e in ((s, e) for s in range(len(self.ep)) for e in range(self.cfg.num_experts)):
            n = int(recv_counts[src, e])
            if n == 0:
                continue
            if e not in self.local_experts:
                raise RuntimeError(f"{self.me} received tokens for expert {e} it does not host")
            w1, w2 = (self.params[_expert_key(e, m)] for m in _EXPERT_MATS)
            outputs.append(expert_ffn(recv[at:at + n], w1, w2))
            at += n
        return torch.cat(outputs) if outputs else recv.new_zeros((0, self.cfg.hidden))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        chosen, gates = route(cfg, x, self.params["router.weight"], self.buffers.get("router.expert_bias"))
        self.tokens_per_expert = torch.bincount(chosen.flatten(), minlength=cfg.num_experts).to(torch.float64)
        tok, slot, counts = self._pack(chosen, self._destinations(chosen))
        group = self.comms.group(f"ep/{self.gidx}")
        recv_counts = _exchange(torch.empty_like(counts), counts, None, None, group, self.wait)
        sent, got = counts.sum(1).tolist(), recv_counts.sum(1).tolist()
        recv = _AllToAll.apply(x.index_select(0, tok), got, sent, group, self.wait)
        back = _AllToAll.apply(self._run_experts(recv, recv_counts), sent, got, group, self.wait)
        return x + torch.zeros_like(x).index_add(0, tok, gates[tok, slot, None] * back)

    def global_loads(self) -> list[float]:
        """Tokens routed to each expert in the last forward, summed over the data-parallel ranks."""
        loads = self.tokens_per_expert.clone()
        group = self.comms.group("dp")
        if group is not None:
            self.wait(dist.all_reduce(loads, group=group, async_op=True))
        return loads.tolist()

    def finish_iteration(self) -> None:
        bias = self.buffers.get("router.expert_bias")
        if bias is not None:
            update_expert_bias(self.cfg, bias, torch.tensor(self.global_loads(), dtype=bias.dtype))

    def _reduce(self, group_name: str, keys: list[str]) -> None:
        group = self.comms.group(group_name)
        if group is None:
            return
        grads = [self.params[k].grad if self.params[k].grad is not None else torch.zeros_like(self.params[k])
                 for k in keys]
        flat = torch.cat([g.reshape(-1) for g in grads])
        self.wait(dist.all_reduce(flat, group=group, async_op=True))
        for k, piece in zip(keys, flat.split([self.params[k].numel() for k in keys])):
            self.params[k].grad = piece.view_as(self.params[k]).clone()

    def sync_grads(self) -> None:
        """Router gradient over all ranks; every replicated expert's over its holders."""
        self._reduce("dp", ["router.weight"])
        for holders, experts in sorted(expert_dp_groups(self.placement).items()):
            if self.me in holders and len(holders) > 1:
                self._reduce(edp_group_name(holders), [_expert_key(e, m) for e in experts for m in _EXPERT_MATS])


def local_keys(placement: ExpertPlacement, me: str, specs: dict[str, TensorSpec]) -> list[str]:
    """The keys ``me`` holds: every dense key and its experts' keys."""
    hosted = set(placement.slots[me])
    return [k for k in specs if expert_of(k) is None or expert_of(k) in hosted]
