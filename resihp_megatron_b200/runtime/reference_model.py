"""The executable float64 reference model: the CPU semantics oracle of the hybrid runtime.

A stack of pre-LN MLP blocks, ``x + fc2(gelu(fc1(LN(x)))) + fc2.bias``, laid out for tensor
parallelism: fc1 column-parallel (dim 0), fc2 row-parallel (dim 1), the LN parameters and
fc2.bias replicated, shards cut by ``even_split`` (uneven shards and any TP degree allowed).
With sequence parallelism the token dimension is sharded between blocks: an all-gather before
fc1 and a reduce-scatter after fc2, each with its autograd transpose.  Parameters are a pure
function of ``(seed, layer)`` and samples of ``(seed, index)``, so every TP degree and pipeline
partition trains the same model on the same data, and any distributed execution can be checked
against ``reference_train``.

Optional fp8-style delayed scaling (``amax_history > 0``) divides the fc1 input by
``1 + 0.1 * max(history)`` and records the iteration's amax: a non-trainable buffer that must
migrate and roll back with its layer.
Parity: ``resihp/runtime/reference_model.py:27-332`` (the same model, so results compare); the
GPT decoder oracle of the GPU benchmark configs is ``reference_gpt.py``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..state.rng_data import IndexAddressableSampler, derive_seed, generator
from ..utils.intervals import even_split

# TP partition dimension of each block parameter (None: replicated)
PARAM_DIMS = {"ln.weight": None, "ln.bias": None, "fc1.weight": 0, "fc1.bias": 0, "fc2.weight": 1, "fc2.bias": None}
# replicated parameters whose gradient is a partial sum over token shards under sequence parallelism
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
    """The unsharded parameters of ``layer`` (drawn in a fixed order from its own generator)."""
    g = generator(cfg.seed, layer, 7)
    h, f = cfg.hidden, cfg.ffn

    def normal(*shape, scale=1.0):
        return scale * torch.randn(*shape, generator=g, dtype=cfg.dtype)

    out = {"ln.weight": 1.0 + normal(h, scale=0.1), "ln.bias": normal(h, scale=0.1)}
    out["fc1.weight"] = normal(f, h) / h ** 0.5
    out["fc1.bias"] = normal(f, scale=0.1)
    out["fc2.weight"] = normal(h, f) / f ** 0.5
    out["fc2.bias"] = normal(h, scale=0.1)
    return out


def shard(t: torch.Tensor, dim: int | None, tp_rank: int, tp_size: int) -> torch.Tensor:
    """TP rank ``tp_rank``'s copy of ``t`` (a clone; the whole tensor when replicated)."""
    if dim is None:
        return t.clone()
    lo, hi = even_split(t.shape[dim], tp_size)[tp_rank]
    return t.narrow(dim, lo, hi - lo).clone()


def sample(cfg: RefModelConfig, index: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Document ``index``: ``seq_min..seq_max`` random tokens and its target ``tanh(x @ T)`` for a
    fixed random teacher ``T``."""
    g = generator(cfg.seed, index, 11)
    length = cfg.seq_min + int(torch.randint(0, cfg.seq_max - cfg.seq_min + 1, (1,), generator=g).item())
    x = torch.randn(length, cfg.hidden, generator=g, dtype=cfg.dtype)
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
    """The documents of micro-batch ``mb``, packed along tokens and zero-padded to a multiple of
    ``token_multiple`` (so every TP degree splits the token dimension)."""
    docs = [sample(cfg, i) for i in sampler.microbatch_indices(iteration, mb)]
    real = sum(x.shape[0] for x, _ in docs)
    padded = -(-real // cfg.token_multiple) * cfg.token_multiple
    x = torch.zeros(padded, cfg.hidden, dtype=cfg.dtype)
    y = torch.zeros(padded, cfg.hidden, dtype=cfg.dtype)
    torch.cat([d[0] for d in docs], out=x[:real])
    torch.cat([d[1] for d in docs], out=y[:real])
    mask = (torch.arange(padded) < real).to(cfg.dtype)
    return MicroBatch(x, y, mask, [d[0].shape[0] for d in docs])


def global_tokens(cfg: RefModelConfig, sampler: IndexAddressableSampler, iteration: int) -> int:
    return sum(sample(cfg, i)[0].shape[0] for i in sampler.batch_indices(iteration))


def token_loss(out: torch.Tensor, y: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Sum over real tokens of the per-token mean squared error."""
    per_token = (out - y).pow(2).mean(dim=-1)
    return (per_token * mask).sum()


# ---------------------------------------------------------------------- tensor-parallel plumbing
Waiter = Callable[[object], None]


class TPContext:
    """The collectives of one TP group; ``waiter`` is the comm manager's abortable wait."""

    def __init__(self, group=None, rank: int = 0, size: int = 1, sequence_parallel: bool = False,
                 waiter: Waiter | None = None):
        self.group, self.rank, self.size = group, rank, size
        self.sequence_parallel = size > 1 and sequence_parallel
        self.waiter = waiter if waiter is not None else (lambda work: work.wait())

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            self.waiter(dist.all_reduce(t, group=self.group, async_op=True))
        return t

    def gather_tokens(self, part: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return part
        pieces = [torch.empty_like(part) for _ in range(self.size)]
        self.waiter(dist.all_gather(pieces, part.contiguous(), group=self.group, async_op=True))
        return torch.cat(pieces)

    def scatter_tokens(self, full: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return full
        lo, hi = even_split(full.shape[0], self.size)[self.rank]
        return full[lo:hi].contiguous()

    def reduce_scatter_tokens(self, full: torch.Tensor) -> torch.Tensor:
        """Reduce-scatter as all-reduce + narrow: the sum order is the all-reduce's."""
        return self.scatter_tokens(self.all_reduce(full.contiguous().clone()))

    # the forward / backward pair of each TP boundary (Megatron's f / g and their SP forms)
    def identity(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def all_reduce_copy(self, t: torch.Tensor) -> torch.Tensor:
        return self.all_reduce(t.contiguous().clone())


class _Boundary(torch.autograd.Function):
    """A TP boundary: ``forward(x) = fwd(x)``, ``backward(g) = bwd(g)`` for two TPContext
    methods named by the caller."""

    @staticmethod
    def forward(ctx, x, tp, fwd: str, bwd: str):
        ctx.tp, ctx.bwd = tp, bwd
        y = getattr(tp, fwd)(x)
        return x.view_as(x) if y is x else y

    @staticmethod
    def backward(ctx, g):
        return getattr(ctx.tp, ctx.bwd)(g.contiguous()), None, None, None


# (forward, backward) at the entry of a column-parallel layer and the exit of a row-parallel one
_ENTER = {"sp": ("gather_tokens", "reduce_scatter_tokens"), "tp": ("identity", "all_reduce_copy")}
_LEAVE = {"sp": ("reduce_scatter_tokens", "gather_tokens"), "tp": ("all_reduce_copy", "identity")}


def _cross(table, h: torch.Tensor, tp: TPContext) -> torch.Tensor:
    if tp.sequence_parallel:
        return _Boundary.apply(h, tp, *table["sp"])
    if tp.size > 1:
        return _Boundary.apply(h, tp, *table["tp"])
    return h


def enter_tp(h: torch.Tensor, tp: TPContext) -> torch.Tensor:
    return _cross(_ENTER, h, tp)


def leave_tp(o: torch.Tensor, tp: TPContext) -> torch.Tensor:
    return _cross(_LEAVE, o, tp)


class RefBlock(torch.nn.Module):
    def __init__(self, cfg: RefModelConfig, layer: int, tp: TPContext):
        super().__init__()
        self.layer, self.tp = layer, tp
        mine = {name: shard(t, PARAM_DIMS[name], tp.rank, tp.size).to(cfg.device)
                for name, t in full_layer_params(cfg, layer).items()}
        self.params = torch.nn.ParameterDict({name.replace(".", "_"): torch.nn.Parameter(t)
                                              for name, t in mine.items()})
        self.fp8 = cfg.amax_history > 0
        if self.fp8:
            self.register_buffer("amax_history", torch.ones(cfg.amax_history, dtype=cfg.dtype, device=cfg.device))
            self.register_buffer("pending_amax", torch.zeros((), dtype=cfg.dtype, device=cfg.device))

    def p(self, name: str) -> torch.nn.Parameter:
        return self.params[name.replace(".", "_")]

    def finish_iteration(self, amax: torch.Tensor) -> None:
        """Delayed-scaling update with the iteration's global amax (MAX over every rank)."""
        with torch.no_grad():
            self.amax_history.copy_(torch.roll(self.amax_history, 1))
            self.amax_history[0] = amax.reshape(())
            self.pending_amax.zero_()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        p = self.p
        normed = F.layer_norm(x, (x.shape[-1],), p("ln.weight"), p("ln.bias"))
        h = enter_tp(normed, self.tp)
        if self.fp8:
            h = h / (1.0 + 0.1 * self.amax_history.max())
            with torch.no_grad():
                torch.maximum(self.pending_amax, h.detach().abs().max(), out=self.pending_amax)
        partial = F.linear(F.gelu(F.linear(h, p("fc1.weight"), p("fc1.bias"))), p("fc2.weight"))
        return x + leave_tp(partial, self.tp) + p("fc2.bias")


def _suffix(key: str) -> str:
    """``layers.<l>.fc1.weight`` -> ``fc1.weight``."""
    return key.split(".", 2)[2]


class RefStage(torch.nn.Module):
    """Layers ``[start, end)`` of the reference model on one TP rank."""

    def __init__(self, cfg: RefModelConfig, start: int, end: int, tp: TPContext | None = None):
        super().__init__()
        self.cfg, self.start, self.end = cfg, start, end
        self.tp = tp if tp is not None else TPContext()
        self.blocks = torch.nn.ModuleList([RefBlock(cfg, layer, self.tp) for layer in range(start, end)])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for block in self.blocks:
            x = block(x)
        return x

    def named_state(self) -> dict[str, torch.nn.Parameter]:
        """Keys independent of stage boundaries: ``layers.<global layer>.<param>``."""
        return {f"layers.{b.layer}.{name}": b.p(name) for b in self.blocks for name in PARAM_DIMS}

    def named_buffer_state(self) -> dict[str, torch.Tensor]:
        return {f"layers.{b.layer}.amax_history": b.amax_history for b in self.blocks if b.fp8}

    def transaction_buffers(self) -> dict[str, torch.Tensor]:
        bufs = self.named_buffer_state()
        for b in (b for b in self.blocks if b.fp8):
            bufs[f"layers.{b.layer}.pending_amax"] = b.pending_amax
        return bufs

    @staticmethod
    def param_dim(key: str) -> int | None:
        return PARAM_DIMS[_suffix(key)]

    def sp_partial(self, key: str) -> bool:
        return self.tp.sequence_parallel and _suffix(key) in SP_PARTIAL


class ChunkedStage(torch.nn.Module):
    """The model chunks of one device under interleaved pipelining (virtual stage -> RefStage),
    with the state interface of a single ``RefStage``."""

    def __init__(self, chunks: dict[int, RefStage]):
        super().__init__()
        self.chunks = {s: chunks[s] for s in sorted(chunks)}
        self._mods = torch.nn.ModuleDict({str(s): m for s, m in self.chunks.items()})
        self.tp = next(iter(self.chunks.values())).tp

    @property
    def blocks(self) -> list[RefBlock]:
        return [b for stage in self.chunks.values() for b in stage.blocks]

    def _merged(self, method: str) -> dict:
        merged = {}
        for stage in self.chunks.values():
            merged.update(getattr(stage, method)())
        return merged

    def named_state(self):
        return self._merged("named_state")

    def named_buffer_state(self):
        return self._merged("named_buffer_state")

    def transaction_buffers(self):
        return self._merged("transaction_buffers")

    param_dim = staticmethod(RefStage.param_dim)

    def sp_partial(self, key: str) -> bool:
        return self.tp.sequence_parallel and _suffix(key) in SP_PARTIAL


def reference_train(cfg: RefModelConfig, sampler: IndexAddressableSampler, iterations: int, lr: float = 1e-2,
                    weight_decay: float = 0.0) -> tuple[list[float], dict[str, torch.Tensor]]:
    """Single-process ground truth: the full model and global batch, loss per global token."""
    from .optim import Adam

    model = RefStage(cfg, 0, cfg.num_layers)
    params = model.named_state()
    opt = Adam(params, lr=lr, weight_decay=weight_decay)
    history = []
    for it in range(iterations):
        opt.zero_grad()
        tokens = global_tokens(cfg, sampler, it)
        total = 0.0
        for mb in range(sampler.num_microbatches):
            batch = microbatch(cfg, sampler, it, mb)
            loss = token_loss(model(batch.x), batch.y, batch.mask)
            (loss / tokens).backward()
            total += loss.item()
        for block in (b for b in model.blocks if b.fp8):
            block.finish_iteration(block.pending_amax.clone())
        opt.step()
        history.append(total / tokens)
    final = {k: v.detach().clone() for k, v in params.items()}
    final.update((k, v.clone()) for k, v in model.named_buffer_state().items())
    return history, final


def init_seed(cfg: RefModelConfig) -> int:
    return derive_seed(cfg.seed, 99)
