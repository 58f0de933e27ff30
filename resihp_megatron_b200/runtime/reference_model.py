"""Executable float64 reference model: the CPU semantics oracle of the runtime.

A stack of pre-LN MLP blocks ``x + fc2(gelu(fc1(LN(x)))) + fc2.bias`` laid out like tensor
parallelism: fc1 column-parallel (dim 0), fc2 row-parallel (dim 1), LN and fc2.bias replicated,
shards from ``even_split`` (uneven shards allowed, any TP degree).  With sequence parallelism the
token dimension is sharded between blocks: all-gather before fc1, reduce-scatter after fc2
(both with their autograd transposes).  Parameters are a pure function of ``(seed, layer)`` and
samples of ``(seed, index)``, so every TP degree and pipeline partition sees the same model and
data, and any distributed execution can be checked against ``reference_train``.

Optional FP8-style delayed scaling (``amax_history > 0``) scales the fc1 input by
``1 / (1 + 0.1 * max(history))`` and records the iteration's global amax -- a non-trainable
buffer that must migrate and roll back with its layer.  (Reference:
``resihp/runtime/reference_model.py:27-332``; the GPT decoder oracle is ``reference_gpt.py``.)
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..state.rng_data import IndexAddressableSampler, derive_seed, generator
from ..utils.intervals import even_split

PARAM_DIMS = {"ln.weight": None, "ln.bias": None, "fc1.weight": 0, "fc1.bias": 0, "fc2.weight": 1, "fc2.bias": None}
SP_PARTIAL = {"ln.weight", "ln.bias", "fc2.bias"}


@dataclass(frozen=True)
class RefModelConfig:
    hidden: int = 8
    ffn: int = 24
    num_layers: int = 4
    seq_min: int = 2
    seq_max: int = 9
    token_multiple: int = 12
    seed: int = 1234
    dtype: torch.dtype = torch.float64
    device: str = "cpu"
    amax_history: int = 0


def full_layer_params(cfg: RefModelConfig, layer: int) -> dict[str, torch.Tensor]:
    g = generator(cfg.seed, layer, 7)
    h, f, dt = cfg.hidden, cfg.ffn, cfg.dtype
    return {
        "ln.weight": 1.0 + 0.1 * torch.randn(h, generator=g, dtype=dt),
        "ln.bias": 0.1 * torch.randn(h, generator=g, dtype=dt),
        "fc1.weight": torch.randn(f, h, generator=g, dtype=dt) / h ** 0.5,
        "fc1.bias": 0.1 * torch.randn(f, generator=g, dtype=dt),
        "fc2.weight": torch.randn(h, f, generator=g, dtype=dt) / f ** 0.5,
        "fc2.bias": 0.1 * torch.randn(h, generator=g, dtype=dt),
    }


def shard(t: torch.Tensor, dim: int | None, tp_rank: int, tp_size: int) -> torch.Tensor:
    if dim is None:
        return t.clone()
    a, b = even_split(t.shape[dim], tp_size)[tp_rank]
    return t.narrow(dim, a, b - a).clone()


def sample(cfg: RefModelConfig, index: int) -> tuple[torch.Tensor, torch.Tensor]:
    """A variable-length document (``seq_min..seq_max`` tokens) and its teacher target."""
    g = generator(cfg.seed, index, 11)
    n = cfg.seq_min + int(torch.randint(0, cfg.seq_max - cfg.seq_min + 1, (1,), generator=g).item())
    x = torch.randn(n, cfg.hidden, generator=g, dtype=cfg.dtype)
    teacher = torch.randn(cfg.hidden, cfg.hidden, generator=generator(cfg.seed, 3), dtype=cfg.dtype)
    return x, torch.tanh(x @ teacher)


@dataclass
class MicroBatch:
    x: torch.Tensor
    y: torch.Tensor
    mask: torch.Tensor
    doc_lengths: list[int]

    @property
    def num_tokens(self) -> int:
        return int(self.mask.sum().item())


def microbatch(cfg: RefModelConfig, sampler: IndexAddressableSampler, iteration: int, mb: int) -> MicroBatch:
    """Documents of micro-batch ``mb`` packed along tokens and padded to ``token_multiple``."""
    xs, ys, lens = [], [], []
    for idx in sampler.microbatch_indices(iteration, mb):
        x, y = sample(cfg, idx)
        xs.append(x)
        ys.append(y)
        lens.append(x.shape[0])
    x, y = torch.cat(xs), torch.cat(ys)
    real = x.shape[0]
    pad = -(-real // cfg.token_multiple) * cfg.token_multiple - real
    mask = torch.cat([torch.ones(real, dtype=cfg.dtype), torch.zeros(pad, dtype=cfg.dtype)])
    x = torch.cat([x, torch.zeros(pad, cfg.hidden, dtype=cfg.dtype)])
    y = torch.cat([y, torch.zeros(pad, cfg.hidden, dtype=cfg.dtype)])
    return MicroBatch(x, y, mask, lens)


def global_tokens(cfg: RefModelConfig, sampler: IndexAddressableSampler, iteration: int) -> int:
    return sum(sample(cfg, i)[0].shape[0] for i in sampler.batch_indices(iteration))


def token_loss(out: torch.Tensor, y: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Sum over real tokens of the per-token mean squared error."""
    return (((out - y) ** 2).mean(dim=-1) * mask).sum()


# ---------------------------------------------------------------------- tensor-parallel plumbing
Waiter = Callable[[object], None]


class TPContext:
    """Collectives of one TP group; ``waiter`` is the abortable wait of the comm manager."""

    def __init__(self, group=None, rank: int = 0, size: int = 1, sequence_parallel: bool = False,
                 waiter: Waiter | None = None):
        self.group = group
        self.rank = rank
        self.size = size
        self.sequence_parallel = sequence_parallel and size > 1
        self.waiter = waiter or (lambda w: w.wait())

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            self.waiter(dist.all_reduce(t, group=self.group, async_op=True))
        return t

    def gather_tokens(self, part: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return part
        bufs = [torch.empty_like(part) for _ in range(self.size)]
        self.waiter(dist.all_gather(bufs, part.contiguous(), group=self.group, async_op=True))
        return torch.cat(bufs)

    def scatter_tokens(self, full: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return full
        a, b = even_split(full.shape[0], self.size)[self.rank]
        return full.narrow(0, a, b - a).contiguous()

    def reduce_scatter_tokens(self, full: torch.Tensor) -> torch.Tensor:
        return self.scatter_tokens(self.all_reduce(full.contiguous().clone()))


class _CopyToTP(torch.autograd.Function):
    """Identity forward, all-reduce backward (input of a column-parallel layer)."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.all_reduce(g.contiguous().clone()), None


class _ReduceFromTP(torch.autograd.Function):
    """All-reduce forward, identity backward (output of a row-parallel layer)."""

    @staticmethod
    def forward(ctx, x, tp):
        return tp.all_reduce(x.contiguous().clone())

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherFromSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.gather_tokens(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.reduce_scatter_tokens(g), None


class _ReduceScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.reduce_scatter_tokens(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.gather_tokens(g.contiguous()), None


def enter_tp(h: torch.Tensor, tp: TPContext) -> torch.Tensor:
    if tp.sequence_parallel:
        return _GatherFromSP.apply(h, tp)
    if tp.size > 1:
        return _CopyToTP.apply(h, tp)
    return h


def leave_tp(o: torch.Tensor, tp: TPContext) -> torch.Tensor:
    if tp.sequence_parallel:
        return _ReduceScatterToSP.apply(o, tp)
    if tp.size > 1:
        return _ReduceFromTP.apply(o, tp)
    return o


class RefBlock(torch.nn.Module):
    def __init__(self, cfg: RefModelConfig, layer: int, tp: TPContext):
        super().__init__()
        self.layer = layer
        self.tp = tp
        full = full_layer_params(cfg, layer)
        self.params = torch.nn.ParameterDict(
            {k.replace(".", "_"): torch.nn.Parameter(shard(v, PARAM_DIMS[k], tp.rank, tp.size).to(cfg.device))
             for k, v in full.items()})
        self.fp8 = cfg.amax_history > 0
        if self.fp8:
            self.register_buffer("amax_history", torch.ones(cfg.amax_history, dtype=cfg.dtype, device=cfg.device))
            self.register_buffer("pending_amax", torch.zeros((), dtype=cfg.dtype, device=cfg.device))

    def p(self, name: str) -> torch.nn.Parameter:
        return self.params[name.replace(".", "_")]

    def finish_iteration(self, amax: torch.Tensor) -> None:
        """Delayed-scaling update with the iteration's global amax (reduced over every rank)."""
        with torch.no_grad():
            self.amax_history.copy_(torch.cat([amax.reshape(1), self.amax_history[:-1]]))
            self.pending_amax.zero_()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = enter_tp(F.layer_norm(x, (x.shape[-1],), self.p("ln.weight"), self.p("ln.bias")), self.tp)
        if self.fp8:
            h = h / (1.0 + 0.1 * self.amax_history.max())
            with torch.no_grad():
                self.pending_amax.copy_(torch.maximum(self.pending_amax, h.detach().abs().max()))
        o = F.linear(F.gelu(F.linear(h, self.p("fc1.weight"), self.p("fc1.bias"))), self.p("fc2.weight"))
        return x + leave_tp(o, self.tp) + self.p("fc2.bias")


class RefStage(torch.nn.Module):
    """Layers ``[start, end)`` of the reference model on one TP rank."""

    def __init__(self, cfg: RefModelConfig, start: int, end: int, tp: TPContext | None = None):
        super().__init__()
        self.cfg = cfg
        self.start, self.end = start, end
        self.tp = tp or TPContext()
        self.blocks = torch.nn.ModuleList(RefBlock(cfg, l, self.tp) for l in range(start, end))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for b in self.blocks:
            x = b(x)
        return x

    def named_state(self) -> dict[str, torch.nn.Parameter]:
        """Keys independent of stage boundaries: ``layers.<global layer>.<param>``."""
        return {f"layers.{b.layer}.{k}": b.p(k) for b in self.blocks for k in PARAM_DIMS}

    def named_buffer_state(self) -> dict[str, torch.Tensor]:
        return {f"layers.{b.layer}.amax_history": b.amax_history for b in self.blocks if b.fp8}

    def transaction_buffers(self) -> dict[str, torch.Tensor]:
        out = dict(self.named_buffer_state())
        out.update({f"layers.{b.layer}.pending_amax": b.pending_amax for b in self.blocks if b.fp8})
        return out

    @staticmethod
    def param_dim(key: str) -> int | None:
        return PARAM_DIMS[key.split(".", 2)[2]]

    def sp_partial(self, key: str) -> bool:
        return self.tp.sequence_parallel and key.split(".", 2)[2] in SP_PARTIAL


class ChunkedStage(torch.nn.Module):
    """The model chunks of one device under interleaved pipelining (virtual stage -> RefStage),
    with the same state interface as one ``RefStage``."""

    def __init__(self, chunks: dict[int, RefStage]):
        super().__init__()
        self.chunks = dict(sorted(chunks.items()))
        self._mods = torch.nn.ModuleDict({str(s): m for s, m in self.chunks.items()})
        self.tp = next(iter(self.chunks.values())).tp

    @property
    def blocks(self) -> list[RefBlock]:
        return [b for m in self.chunks.values() for b in m.blocks]

    def named_state(self):
        return {k: v for m in self.chunks.values() for k, v in m.named_state().items()}

    def named_buffer_state(self):
        return {k: v for m in self.chunks.values() for k, v in m.named_buffer_state().items()}

    def transaction_buffers(self):
        return {k: v for m in self.chunks.values() for k, v in m.transaction_buffers().items()}

    param_dim = staticmethod(RefStage.param_dim)

    def sp_partial(self, key: str) -> bool:
        return self.tp.sequence_parallel and key.split(".", 2)[2] in SP_PARTIAL


def reference_train(cfg: RefModelConfig, sampler: IndexAddressableSampler, iterations: int, lr: float = 1e-2,
                    weight_decay: float = 0.0) -> tuple[list[float], dict[str, torch.Tensor]]:
    """Single-process ground truth: full model, full global batch, loss per global token."""
    from .optim import Adam

    model = RefStage(cfg, 0, cfg.num_layers)
    params = model.named_state()
    opt = Adam(params, lr=lr, weight_decay=weight_decay)
    losses = []
    for it in range(iterations):
        opt.zero_grad()
        total = global_tokens(cfg, sampler, it)
        loss_sum = 0.0
        for mb in range(sampler.num_microbatches):
            m = microbatch(cfg, sampler, it, mb)
            l = token_loss(model(m.x), m.y, m.mask)
            (l / total).backward()
            loss_sum += l.item()
        for b in model.blocks:
            if b.fp8:
                b.finish_iteration(b.pending_amax.clone())
        opt.step()
        losses.append(loss_sum / total)
    state = {k: v.detach().clone() for k, v in params.items()}
    state.update({k: v.clone() for k, v in model.named_buffer_state().items()})
    return losses, state


def init_seed(cfg: RefModelConfig) -> int:
    return derive_seed(cfg.seed, 99)
