"""Float64 GPT decoder: the CPU oracle of the decoder architecture the GPU model runs.

Same architecture as ``models/gpt.py`` -- token embedding, pre-norm RMSNorm, causal multi-head
attention with grouped KV heads and rotary embeddings, SwiGLU MLP, untied LM head, token
cross-entropy -- written with plain autograd tensor ops in float64 on the CPU.  It serves
(a) the CPU/gloo resilience config (DP over worker processes, bit-identical loss after a
``kill -9``) and (b) numerical cross-checks of the GPU kernels.

Parameters are drawn ``N(0, init_std)`` from ``generator(seed, param-name hash)``, so every
process builds the same model; synthetic batches are uniform token ids from
``generator(data_seed, iteration, micro-batch)``, a pure function of the micro-batch identity.
``train_single_process`` accumulates per-micro-batch gradients in micro-batch order and divides
by the global token count at the end -- the exact arithmetic of the canonical DP reduction, so
a DP run of any size (or one reconfigured mid-run) is bitwise equal to it.
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass

import torch

from ..state.rng_data import generator


@dataclass(frozen=True)
class GPTRefConfig:
    vocab: int = 512
    hidden: int = 64
    layers: int = 4
    heads: int = 4
    kv_heads: int = 4
    ffn: int = 256
    seq: int = 32
    micro_batch: int = 2
    num_microbatches: int = 8
    init_std: float = 0.02
    seed: int = 0          # parameter seed
    data_seed: int = 1     # token seed
    rope_theta: float = 10000.0
    eps: float = 1e-5
    dtype: torch.dtype = torch.float64

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def tokens_per_iteration(self) -> int:
        return self.num_microbatches * self.micro_batch * self.seq


def _key_seed(name: str) -> int:
    return int.from_bytes(hashlib.sha256(name.encode()).digest()[:4], "little")


def param_shapes(cfg: GPTRefConfig) -> dict[str, tuple[int, ...]]:
    H, D, F = cfg.hidden, cfg.head_dim, cfg.ffn
    shapes = {"embed": (cfg.vocab, H)}
    for l in range(cfg.layers):
        p = f"layers.{l}."
        shapes.update({p + "attn_norm": (H,), p + "wq": (cfg.heads * D, H), p + "wk": (cfg.kv_heads * D, H),
                       p + "wv": (cfg.kv_heads * D, H), p + "wo": (H, cfg.heads * D), p + "mlp_norm": (H,),
                       p + "w1": (F, H), p + "w3": (F, H), p + "w2": (H, F)})
    shapes.update({"final_norm": (H,), "lm_head": (cfg.vocab, H)})
    return shapes


def init_params(cfg: GPTRefConfig) -> dict[str, torch.Tensor]:
    out = {}
    for name, shape in param_shapes(cfg).items():
        if name.endswith("norm"):
            out[name] = torch.ones(shape, dtype=cfg.dtype)
        else:
            g = generator(cfg.seed, _key_seed(name))
            out[name] = torch.randn(shape, generator=g, dtype=cfg.dtype) * cfg.init_std
    return out


def batch(cfg: GPTRefConfig, iteration: int, mb: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Token ids ``[micro_batch, seq]`` and next-token labels for (iteration, micro-batch)."""
    g = generator(cfg.data_seed, iteration, mb)
    seq = torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq + 1), generator=g)
    return seq[:, :-1], seq[:, 1:]


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half RoPE on [B, S, heads, D]."""
    B, S, Hh, D = x.shape
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=x.dtype) / D))
    ang = torch.outer(torch.arange(S, dtype=x.dtype), inv)
    cos = ang.cos().repeat(1, 2).view(1, S, 1, D)
    sin = ang.sin().repeat(1, 2).view(1, S, 1, D)
    rot = torch.cat([-x[..., D // 2:], x[..., : D // 2]], -1)
    return x * cos + rot * sin


def forward_loss(cfg: GPTRefConfig, P: dict[str, torch.Tensor], ids: torch.Tensor, labels: torch.Tensor,
                 layers: range | None = None) -> torch.Tensor:
    """Summed token cross-entropy of one micro-batch."""
    B, S = ids.shape
    H, D, Hq, Hk = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
    x = P["embed"][ids.reshape(-1)].view(B, S, H)
    mask = torch.ones(S, S, dtype=torch.bool).triu(1)
    for l in (layers if layers is not None else range(cfg.layers)):
        p = f"layers.{l}."
        h = _rms(x, P[p + "attn_norm"], cfg.eps)
        q = _rope((h @ P[p + "wq"].t()).view(B, S, Hq, D), cfg.rope_theta).transpose(1, 2)
        k = _rope((h @ P[p + "wk"].t()).view(B, S, Hk, D), cfg.rope_theta).transpose(1, 2)
        v = (h @ P[p + "wv"].t()).view(B, S, Hk, D).transpose(1, 2)
        if Hk != Hq:
            k = k.repeat_interleave(Hq // Hk, 1)
            v = v.repeat_interleave(Hq // Hk, 1)
        att = (q @ k.transpose(-1, -2)) / math.sqrt(D)
        att = att.masked_fill(mask, float("-inf")).softmax(-1)
        o = (att @ v).transpose(1, 2).reshape(B, S, Hq * D)
        x = x + o @ P[p + "wo"].t()
        h2 = _rms(x, P[p + "mlp_norm"], cfg.eps)
        a = torch.nn.functional.silu(h2 @ P[p + "w1"].t()) * (h2 @ P[p + "w3"].t())
        x = x + a @ P[p + "w2"].t()
    logits = _rms(x, P["final_norm"], cfg.eps) @ P["lm_head"].t()
    return torch.nn.functional.cross_entropy(logits.reshape(B * S, cfg.vocab), labels.reshape(-1), reduction="sum")


class GPTRefModel:
    """Holds float64 parameters (``named_state``) for the DP runtime and the bindings."""

    def __init__(self, cfg: GPTRefConfig):
        self.cfg = cfg
        self.params = {k: v.requires_grad_(True) for k, v in init_params(cfg).items()}

    def named_state(self) -> dict[str, torch.Tensor]:
        return self.params

    def loss(self, ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return forward_loss(self.cfg, self.params, ids, labels)


def microbatch_grads(cfg: GPTRefConfig, params: dict[str, torch.Tensor], iteration: int, mb: int):
    """Flat gradient vector of one micro-batch's summed loss, with the loss appended."""
    ids, labels = batch(cfg, iteration, mb)
    names = list(params)
    loss = forward_loss(cfg, params, ids, labels)
    grads = torch.autograd.grad(loss, [params[n] for n in names])
    return torch.cat([g.reshape(-1) for g in grads] + [loss.detach().reshape(1)])


def train_single_process(cfg: GPTRefConfig, iterations: int, lr: float = 1e-3, betas=(0.9, 0.95),
                         eps: float = 1e-8) -> tuple[list[float], dict[str, torch.Tensor]]:
    """Ground truth for the DP resilience test: canonical micro-batch-order accumulation."""
    from .optim import Adam

    torch.set_num_threads(1)
    model = GPTRefModel(cfg)
    opt = Adam(model.params, lr=lr, betas=betas, eps=eps)
    names = list(model.params)
    losses = []
    total = cfg.tokens_per_iteration
    for it in range(iterations):
        acc = None
        for mb in range(cfg.num_microbatches):
            v = microbatch_grads(cfg, model.params, it, mb)
            acc = v if acc is None else acc + v
        off = 0
        for n in names:
            p = model.params[n]
            p.grad = (acc[off:off + p.numel()].view_as(p) / total).clone()
            off += p.numel()
        opt.step()
        losses.append(acc[-1].item() / total)
    return losses, {k: v.detach().clone() for k, v in model.params.items()}
