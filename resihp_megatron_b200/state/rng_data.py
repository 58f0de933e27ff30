"""Placement-independent data and randomness.

A micro-batch is identified by ``(iteration, global micro-batch id)``.  The samples it holds
and every random number it draws are pure functions of that identity, so it can be executed
again after a failure, or by a different DP replica than planned, without changing what is
trained.  Seeds come from SplitMix64 (Steele, Lea & Flood, "Fast splittable pseudorandom number
generators", OOPSLA 2014) folded over the identity's parts; the sampler takes global batch ``i``
as a fixed window of a per-epoch permutation, independent of the DP size.
Parity: ``resihp/state/rng_data.py:21-112`` (same seeding scheme and sampler contract).
"""

from __future__ import annotations

import functools
import random
from dataclasses import dataclass

import numpy as np
import torch

_MASK64 = (1 << 64) - 1
# SplitMix64's increment and mixing multipliers, as published with the algorithm
_GOLDEN, _MIX1, _MIX2 = 0x9E3779B97F4A7C15, 0xBF58476D1CE4E5B9, 0x94D049BB133111EB


def splitmix64(x: int) -> int:
    """One SplitMix64 output step."""
    z = (x + _GOLDEN) & _MASK64
    for shift, mult in ((30, _MIX1), (27, _MIX2)):
        z = ((z ^ (z >> shift)) * mult) & _MASK64
    return z ^ (z >> 31)


def derive_seed(*parts: int) -> int:
    """A 63-bit seed from a tuple of integers (order matters)."""
    state = functools.reduce(lambda h, p: splitmix64(h ^ (int(p) & _MASK64)), parts, 0)
    return state & (_MASK64 >> 1)


def generator(*parts: int, device: str = "cpu") -> torch.Generator:
    gen = torch.Generator(device=device)
    gen.manual_seed(derive_seed(*parts))
    return gen


class IndexAddressableSampler:
    def __init__(self, num_samples: int, global_batch_size: int, micro_batch_size: int, seed: int = 0,
                 shuffle: bool = True):
        if global_batch_size % micro_batch_size:
            raise ValueError("the global batch must be a multiple of the micro-batch")
        self.num_samples, self.seed, self.shuffle = num_samples, seed, shuffle
        self.global_batch_size, self.micro_batch_size = global_batch_size, micro_batch_size
        self._orders: dict[int, np.ndarray] = {}  # a few recent epochs' permutations

    @property
    def num_microbatches(self) -> int:
        return self.global_batch_size // self.micro_batch_size

    def _order(self, epoch: int) -> np.ndarray:
        if epoch not in self._orders:
            if len(self._orders) >= 4:
                self._orders.pop(next(iter(self._orders)))
            self._orders[epoch] = (np.random.default_rng(derive_seed(self.seed, epoch)).permutation(self.num_samples)
                                   if self.shuffle else np.arange(self.num_samples))
        return self._orders[epoch]

    def sample_index(self, position: int) -> int:
        """The dataset index at a position of the endless, epoch-shuffled stream."""
        epoch, offset = divmod(position, self.num_samples)
        return int(self._order(epoch)[offset])

    def _window(self, start: int, count: int) -> list[int]:
        return [self.sample_index(p) for p in range(start, start + count)]

    def batch_indices(self, iteration: int) -> list[int]:
        return self._window(iteration * self.global_batch_size, self.global_batch_size)

    def microbatch_indices(self, iteration: int, mb: int) -> list[int]:
        if mb < 0 or mb >= self.num_microbatches:
            raise IndexError(mb)
        start = iteration * self.global_batch_size + mb * self.micro_batch_size
        return self._window(start, self.micro_batch_size)

    def consumed_samples(self, iteration: int) -> int:
        return self.global_batch_size * iteration


@dataclass
class DataCursor:
    iteration: int = 0

    def snapshot(self) -> dict:
        return {"iteration": self.iteration}

    def restore(self, snap: dict) -> None:
        self.iteration = snap["iteration"]


def capture_rng_state() -> dict:
    """Every global RNG this process draws from (Python, NumPy, torch CPU, every CUDA device)."""
    state = dict(python=random.getstate(), numpy=np.random.get_state(), torch=torch.get_rng_state())
    if torch.cuda.is_available():
        state["cuda"] = torch.cuda.get_rng_state_all()
    return state


def restore_rng_state(st: dict) -> None:
    random.setstate(st["python"])
    np.random.set_state(st["numpy"])
    torch.set_rng_state(st["torch"])
    if torch.cuda.is_available() and "cuda" in st:
        torch.cuda.set_rng_state_all(st["cuda"])
