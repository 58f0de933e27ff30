"""Placement-independent data and randomness.

A micro-batch is identified by ``(iteration, global micro-batch id)``; the samples it holds and
every random number it draws are pure functions of that identity, so it can be re-executed after
a failure, or by another DP replica than planned, without changing training semantics.
Seeds are derived with SplitMix64 (Steele, Lea & Flood, 2014) chained over the parts; the sampler
takes global batch ``i`` as a fixed slice of a per-epoch permutation, independent of the DP size.
(Reference: ``resihp/state/rng_data.py:21-112``.)
"""

from __future__ import annotations

import random
from dataclasses import dataclass

import numpy as np
import torch

_M64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    """One SplitMix64 output step (published constants of the algorithm)."""
    z = (x + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def derive_seed(*parts: int) -> int:
    h = 0
    for p in parts:
        h = splitmix64(h ^ (int(p) & _M64))
    return h & ((1 << 63) - 1)


def generator(*parts: int, device: str = "cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(derive_seed(*parts))
    return g


class IndexAddressableSampler:
    def __init__(self, num_samples: int, global_batch_size: int, micro_batch_size: int, seed: int = 0,
                 shuffle: bool = True):
        if global_batch_size % micro_batch_size:
            raise ValueError("the global batch must be a multiple of the micro-batch")
        self.num_samples = num_samples
        self.global_batch_size = global_batch_size
        self.micro_batch_size = micro_batch_size
        self.seed = seed
        self.shuffle = shuffle
        self._perms: dict[int, np.ndarray] = {}

    @property
    def num_microbatches(self) -> int:
        return self.global_batch_size // self.micro_batch_size

    def _perm(self, epoch: int) -> np.ndarray:
        p = self._perms.get(epoch)
        if p is None:
            p = (np.random.default_rng(derive_seed(self.seed, epoch)).permutation(self.num_samples)
                 if self.shuffle else np.arange(self.num_samples))
            if len(self._perms) > 4:
                self._perms.clear()
            self._perms[epoch] = p
        return p

    def sample_index(self, position: int) -> int:
        epoch, off = divmod(position, self.num_samples)
        return int(self._perm(epoch)[off])

    def batch_indices(self, iteration: int) -> list[int]:
        base = iteration * self.global_batch_size
        return [self.sample_index(base + i) for i in range(self.global_batch_size)]

    def microbatch_indices(self, iteration: int, mb: int) -> list[int]:
        if not 0 <= mb < self.num_microbatches:
            raise IndexError(mb)
        base = iteration * self.global_batch_size + mb * self.micro_batch_size
        return [self.sample_index(base + i) for i in range(self.micro_batch_size)]

    def consumed_samples(self, iteration: int) -> int:
        return iteration * self.global_batch_size


@dataclass
class DataCursor:
    iteration: int = 0

    def snapshot(self) -> dict:
        return {"iteration": self.iteration}

    def restore(self, snap: dict) -> None:
        self.iteration = snap["iteration"]


def capture_rng_state() -> dict:
    st = {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state()}
    if torch.cuda.is_available():
        st["cuda"] = torch.cuda.get_rng_state_all()
    return st


def restore_rng_state(st: dict) -> None:
    random.setstate(st["python"])
    np.random.set_state(st["numpy"])
    torch.set_rng_state(st["torch"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(st["cuda"])
