"""Flat parameter storage for mixed-precision training.

All trainable tensors of a model shard live in four flat fp32 buffers (master weights,
gradient, Adam first and second moment) plus one flat bf16 buffer (the compute copy the
kernels read).  Each parameter is a view into them, padded to a 64-element boundary so
every view starts on a 256-byte boundary (TMA and vector loads need 16 B).  One fused Adam
launch then updates the whole shard, gradient reduce-scatter works on contiguous buckets,
and migration / checkpointing address a tensor by (offset, numel).

Initialisation is layout invariant: the full logical tensor is drawn from a generator seeded
by ``(seed, name)`` and the shard keeps its slice, so any TP/PP/DP layout starts from the
same weights (the reference achieves the same with counter-based seeds,
``resihp/runtime/reference_model.py:49-59``).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch

ALIGN = 64


@dataclass
class ParamSpec:
    name: str
    shape: tuple[int, ...]           # local (shard) shape
    full_shape: tuple[int, ...] = ()  # logical shape before sharding
    shard_dim: int | None = None      # dimension split across TP ranks (None = replicated)
    shard_range: tuple[int, int] | None = None
    init: str = "normal"              # normal | ones | zeros

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def name_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}/{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


class FlatParams:
    """bf16 compute weights + fp32 master / grad / exp_avg / exp_avg_sq over one flat index space."""

    def __init__(self, specs: list[ParamSpec], device, with_optimizer: bool = True, shard_rank: int = 0,
                 shard_count: int = 1, buffer_factory=None, opt_factory=None):
        """``shard_rank / shard_count`` > 1 keeps the optimizer state (master, moments) for one
        contiguous slice of the flat index space only (ZeRO-1); bf16 weights and gradients stay
        full size.  ``buffer_factory(numel) -> (bf16, grad)`` and ``opt_factory(shard_numel) ->
        (master, exp_avg, exp_avg_sq)`` supply zero-filled flat buffers from elsewhere (the
        symmetric peer heap of the fused data-parallel step, where peers can read them)."""
        self.specs = {s.name: s for s in specs}
        self.order = [s.name for s in specs]
        self.offsets: dict[str, int] = {}
        off = 0
        for s in specs:
            self.offsets[s.name] = off
            off += (s.numel + ALIGN - 1) // ALIGN * ALIGN
        quantum = ALIGN * shard_count
        self.numel = (off + quantum - 1) // quantum * quantum
        self.shard_rank, self.shard_count = shard_rank, shard_count
        self.shard_numel = self.numel // shard_count
        self.shard_lo = shard_rank * self.shard_numel
        self.device = torch.device(device)
        if buffer_factory is not None:
            self.bf16, self.grad = buffer_factory(self.numel)
            assert self.bf16.numel() == self.numel and self.grad.numel() == self.numel
        else:
            self.bf16 = torch.zeros(self.numel, dtype=torch.bfloat16, device=self.device)
            self.grad = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        if with_optimizer and opt_factory is not None:
            self.master, self.exp_avg, self.exp_avg_sq = opt_factory(self.shard_numel)
        elif with_optimizer:
            n = self.shard_numel
            self.master = torch.zeros(n, dtype=torch.float32, device=self.device)
            self.exp_avg = torch.zeros(n, dtype=torch.float32, device=self.device)
            self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=self.device)
        else:
            self.master = self.exp_avg = self.exp_avg_sq = None
        self.step = 0

    @staticmethod
    def flat_numel(specs: list[ParamSpec], shard_count: int) -> int:
        """Padded flat size for ``shard_count`` optimizer shards (what ``__init__`` computes)."""
        off = 0
        for s in specs:
            off += (s.numel + ALIGN - 1) // ALIGN * ALIGN
        quantum = ALIGN * shard_count
        return (off + quantum - 1) // quantum * quantum

    @property
    def sharded(self) -> bool:
        return self.shard_count > 1

    def shard_slice(self, buf: torch.Tensor) -> torch.Tensor:
        """The owned slice of a full-size flat buffer (``bf16`` or ``grad``)."""
        return buf[self.shard_lo:self.shard_lo + self.shard_numel]

    def _view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        s = self.specs[name]
        o = self.offsets[name]
        return buf[o:o + s.numel].view(s.shape)

    def w(self, name: str) -> torch.Tensor:
        return self._view(self.bf16, name)

    def g(self, name: str) -> torch.Tensor:
        return self._view(self.grad, name)

    def m(self, name: str) -> torch.Tensor:
        assert not self.sharded, "master views of a sharded optimizer state are per-slice"
        return self._view(self.master, name)

    def state(self, kind: str, name: str) -> torch.Tensor:
        buf = {"param": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq, "grad": self.grad,
               "bf16": self.bf16}[kind]
        if kind in ("param", "exp_avg", "exp_avg_sq"):
            assert not self.sharded, "use owned_piece() for sharded optimizer state"
        return self._view(buf, name)

    def owned_piece(self, name: str) -> tuple[int, int, int] | None:
        """``(start_in_param, start_in_shard, length)`` of the part of ``name`` this shard owns."""
        o, n = self.offsets[name], self.specs[name].numel
        lo = max(o, self.shard_lo)
        hi = min(o + n, self.shard_lo + self.shard_numel)
        if lo >= hi:
            return None
        return lo - o, lo - self.shard_lo, hi - lo

    @torch.no_grad()
    def initialize(self, seed: int, std: float) -> None:
        """Draw every tensor from its own (seed, name) stream; shards take their slice."""
        for name in self.order:
            s = self.specs[name]
            full = s.full_shape or s.shape
            if s.init == "ones":
                t = torch.ones(full)
            elif s.init == "zeros":
                t = torch.zeros(full)
            else:
                g = torch.Generator(device=self.device).manual_seed(name_seed(seed, name))
                t = torch.empty(full, device=self.device).normal_(0.0, std, generator=g)
            if s.shard_dim is not None and s.shard_range is not None:
                lo, hi = s.shard_range
                t = t.narrow(s.shard_dim, lo, hi - lo)
            t = t.to(self.device, torch.float32).reshape(s.shape)
            if self.master is not None:
                piece = self.owned_piece(name)
                if piece is not None:
                    a, b, n = piece
                    self.master[b:b + n].copy_(t.reshape(-1)[a:a + n])
            self._view(self.bf16, name).copy_(t)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def memory_bytes(self) -> int:
        n = self.numel
        return n * 2 + n * 4 * (4 if self.master is not None else 1)
