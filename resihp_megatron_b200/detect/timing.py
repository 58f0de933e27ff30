"""Per-chunk (F / B / W) timing that never stalls the training stream.

On CUDA every timed chunk is bracketed by two events on the current stream; an event pair is
read back only once the GPU has passed it (typically during the next iteration), so measuring
adds no synchronisation.  On the CPU the wall clock is used, plus the fault injector's compute
padding when one is installed (host-side fail-slow emulation).
Parity: ``resihp/detect/timing.py:25-58`` (same records and deferred readback).
"""

from __future__ import annotations

import time
from collections import deque
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
        self._in_flight: deque = deque()      # (record without time, start event, end event)
        self._ready: list[ChunkRecord] = []

    def _wall(self, iteration: int, op: str, mb: int, started: float) -> None:
        elapsed = time.perf_counter() - started
        if self.injector is not None:
            elapsed += self.injector.pad_compute(elapsed)
        self._ready.append(ChunkRecord(iteration, op, mb, elapsed))

    @contextmanager
    def time(self, iteration: int, op: str, mb: int):
        if not self.use_cuda:
            started = time.perf_counter()
            yield
            self._wall(iteration, op, mb, started)
            return
        begin, end = (torch.cuda.Event(enable_timing=True) for _ in range(2))
        begin.record()
        yield
        end.record()
        self._in_flight.append(((iteration, op, mb), begin, end))

    def collect(self, upto_iteration: int | None = None) -> list[ChunkRecord]:
        """Records finished so far (CUDA pairs whose end event completed, up to an iteration)."""
        waiting = deque()
        while self._in_flight:
            key, begin, end = self._in_flight.popleft()
            eligible = upto_iteration is None or key[0] <= upto_iteration
            if eligible and end.query():
                self._ready.append(ChunkRecord(*key, begin.elapsed_time(end) / 1000.0))
            else:
                waiting.append((key, begin, end))
        self._in_flight = waiting
        done, self._ready = self._ready, []
        return done
