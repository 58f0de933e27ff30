"""Per-chunk (F / B / W) timing with deferred readback.

On CUDA each chunk is bracketed by events that are read back once complete (one iteration
later), so measuring never synchronises the training stream; on the CPU the wall clock is used
and the fault injector's compute padding is added (fail-slow emulation).
(Reference: ``resihp/detect/timing.py:25-58``.)
"""

from __future__ import annotations

import time
from contextlib import contextmanager
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ChunkRecord:
    iteration: int
    op: str
    mb: int
    seconds: float


class ChunkTimer:
    def __init__(self, use_cuda: bool | None = None, injector=None):
        self.use_cuda = torch.cuda.is_available() if use_cuda is None else use_cuda
        self.injector = injector
        self._pending: list[tuple] = []
        self._done: list[ChunkRecord] = []

    @contextmanager
    def time(self, iteration: int, op: str, mb: int):
        if self.use_cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            yield
            b.record()
            self._pending.append((iteration, op, mb, a, b))
        else:
            t0 = time.perf_counter()
            yield
            dt = time.perf_counter() - t0
            if self.injector is not None:
                dt += self.injector.pad_compute(dt)
            self._done.append(ChunkRecord(iteration, op, mb, dt))

    def collect(self, upto_iteration: int | None = None) -> list[ChunkRecord]:
        keep = []
        for it, op, mb, a, b in self._pending:
            if (upto_iteration is None or it <= upto_iteration) and b.query():
                self._done.append(ChunkRecord(it, op, mb, a.elapsed_time(b) / 1e3))
            else:
                keep.append((it, op, mb, a, b))
        self._pending = keep
        out, self._done = self._done, []
        return out
