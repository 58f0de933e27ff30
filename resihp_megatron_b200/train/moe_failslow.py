"""Fail-slow detection for expert parallelism: per-rank expert compute time -> residual BOCD ->
expert re-placement.

``ExpertClock`` times this rank's expert GEMMs of every step (CUDA events around the compute on
GPUs -- the transport's barriers are outside the timed regions, so a straggler does not inflate
its peers' times -- or the wall clock on the CPU) together with the rows they processed.  It can
also emulate a slow GPU from the host: after each timed region it waits for the region's work and
idles ``(slowdown - 1)`` times its duration before closing the region, so the device timeline of
this rank shows the stretch (the duty-cycle injection of the reference's fault injector, with no
device-side injector and no change to any GPU setting).

``ExpertSlowMonitor`` receives every rank's (time, rows) per step, normalises time per row and
takes the median rank as the prediction -- the common-mode normalisation that removes
workload and whole-job swings -- and runs one residual ``FailSlowDetector`` (``log(observed /
predicted)``, BOCD with warm-up calibration) per rank.  A detection yields the rank's relative
speed ``p = predicted / observed`` for the expert-placement planner.
(Reference: ``resihp/detect/failslow.py:36-124`` and ``resihp/plan/expert_placement.py``.)
"""

from __future__ import annotations

import statistics
import time

import torch

from ..detect.failslow import FailSlowDetector


class ExpertClock:
    """``model_ms_per_row``: report a modelled time (rows x cost x slowdown, with 2 % seeded
    jitter) instead of measuring -- for CPU tests of the detection and re-placement logic, whose
    process timings carry far more noise than a GPU's device timeline."""

    def __init__(self, device, slowdown: float = 1.0, model_ms_per_row: float | None = None, seed: int = 0):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.slowdown = float(slowdown)
        self.model = model_ms_per_row
        self._rng = torch.Generator().manual_seed(seed)
        self.regions: list = []  # (start, end, rows) of the current step
        self._open = None

    def begin(self, rows: int) -> None:
        if self.model is not None:
            self._open = (None, rows)
            return
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._open = (ev, rows)
        else:
            self._open = (time.perf_counter(), rows)

    def end(self) -> None:
        start, rows = self._open
        self._open = None
        if self.model is not None:
            jitter = 1.0 + 0.02 * (2.0 * torch.rand((), generator=self._rng).item() - 1.0)
            self.regions.append((0.0, rows * self.model * self.slowdown * jitter / 1000.0, rows))
            return
        if self.cuda:
            if self.slowdown > 1.0:  # idle after the region's work so the device timeline stretches
                stop = torch.cuda.Event(enable_timing=True)
                stop.record()
                stop.synchronize()
                time.sleep((self.slowdown - 1.0) * start.elapsed_time(stop) / 1000.0)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.regions.append((start, ev, rows))
        else:
            if self.slowdown > 1.0:
                time.sleep((self.slowdown - 1.0) * (time.perf_counter() - start))
            self.regions.append((start, time.perf_counter(), rows))

    def collect(self) -> tuple[float, int]:
        """``(milliseconds, rows)`` of the step's expert regions; resets.  On GPUs it waits for
        the last region's end event (the caller has already read the step's loss)."""
        ms, rows = 0.0, 0
        for start, end, n in self.regions:
            if self.cuda and self.model is None:
                end.synchronize()
                ms += start.elapsed_time(end)
            else:
                ms += (end - start) * 1000.0
            rows += n
        self.regions = []
        return ms, rows


class ExpertSlowMonitor:
    def __init__(self, world: int, *, warmup: int = 8, threshold: float = 0.9, window: int = 3,
                 min_increase: float = 0.15, cooldown: int = 10):
        self.world = world
        self.kw = dict(mode="residual", warmup=warmup, threshold=threshold, window=window, min_increase=min_increase,
                       cooldown=cooldown)
        self.detectors = [FailSlowDetector(**self.kw) for _ in range(world)]
        self.history: list[list[float]] = []

    def reset(self) -> None:
        """After a re-placement the per-rank work changes: start the series afresh."""
        self.detectors = [FailSlowDetector(**self.kw) for _ in range(self.world)]

    def observe(self, iteration: int, times_ms: list[float], rows: list[int]) -> dict[int, float]:
        """Every rank's step (same inputs on every rank, so every rank decides the same).
        Returns ``{rank: relative speed}`` for the ranks flagged slow at this step."""
        per = [t / n if n > 0 and t > 0 else None for t, n in zip(times_ms, rows)]
        seen = [p for p in per if p is not None]
        self.history.append(per)
        del self.history[:-256]  # a bounded record of the recent series
        if len(seen) < max(2, self.world // 2 + 1):  # too few ranks did expert work this step
            return {}
        pred = statistics.median(seen)
        out = {}
        for r in range(self.world):
            if per[r] is None:  # no rows routed to this rank's experts: nothing to judge
                continue
            det = self.detectors[r].observe(iteration, per[r], pred)
            if det is not None:
                out[r] = pred / per[r]
        return out
