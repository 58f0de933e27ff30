"""The coordinator-side fail-slow pipeline.

Timing reports arrive one per TP group per iteration (forward-chunk seconds with workload
features).  They are normalised per layer and by TP x CP, fed to one shared gated RLS model, and
each group has its own residual BOCD detector.  A detection gives the group's slowdown ratio;
the ski-rental policy decides whether mitigating it pays, and if so the group's devices get
health ``p = 1 / ratio`` and a replan is requested.  The planner reads ``p`` when it builds the
next plan, so mitigation (TP reshaping, repartition, migration, exclusion) reuses the fail-stop
machinery.  With a ``what_if`` pricer the rent is (current plan - replanned plan) and the price
is the estimated migration + rebuild time, so a slowdown the planner cannot mitigate never
triggers a reconfiguration.

Common-mode correction (``common_mode=True``): an iteration's reports are processed together,
and with three or more groups every group's time is divided by the median observed / predicted
ratio over the groups before reaching its detector and the shared model.  A whole-node slowdown
(contention, a thermal event, a noisy neighbour) moves every group alike and cancels; a
fail-slow device moves only its own group and stands out.
Parity: ``resihp/detect/service.py:30-114`` (same pipeline; the common-mode step is ours).
"""

from __future__ import annotations

import queue
import statistics
import threading
import time
from dataclasses import dataclass, field

from .failslow import FailSlowDetector
from .policy import SkiRentalPolicy
from .predictor import RLSPredictor
from ..utils.log import get_logger

log = get_logger(__name__)


@dataclass
class _Suspect:
    gen: object
    ratio: float
    since: int
    price: tuple | None = None


@dataclass
class _Batcher:
    """Collects an iteration's reports until every group of the generation has reported it (or a
    group is already two iterations ahead)."""

    pending: dict = field(default_factory=dict)   # (gen, iteration) -> {devices: (worker, report)}
    groups: dict = field(default_factory=dict)    # gen -> set of device tuples seen

    def add(self, worker_id: str, report: dict):
        gen, it, devices = report.get("gen"), report["iteration"], tuple(report["devices"])
        members = self.groups.setdefault(gen, set())
        members.add(devices)
        self.pending.setdefault((gen, it), {})[devices] = (worker_id, report)
        for key in sorted(k for k in self.pending if k[0] == gen):
            batch = self.pending[key]
            if set(batch) >= members or key[1] <= it - 2:
                yield list(self.pending.pop(key).values())


class DetectorService:
    def __init__(self, coordinator, *, warmup: int = 6, threshold: float = 0.9, min_increase: float = 0.25,
                 reconfig_cost_s: float = 0.0, min_gain: float = 0.05, min_dwell: int = 0, token_scale: float = 1e3,
                 what_if=None, common_mode: bool = True, window: int = 8):
        self.coord = coordinator
        # a change counts while it lies within the last ``window`` iterations: noisy timings may need
        # several post-change samples before the posterior is confident
        self.detector_kw = dict(mode="residual", warmup=warmup, threshold=threshold, min_increase=min_increase,
                                cooldown=warmup, window=window)
        self.policy_kw = dict(min_gain=min_gain, min_dwell=min_dwell)
        self.rls = RLSPredictor(scales=(token_scale, token_scale ** 2, 1.0), gate=0.3, warmup=32)
        self.detectors: dict[tuple, FailSlowDetector] = {}
        self.policies: dict[tuple, SkiRentalPolicy] = {}
        self.reconfig_cost_s, self.what_if, self.common_mode = reconfig_cost_s, what_if, common_mode
        self.speeds: dict[str, float] = {}
        self.events: list[dict] = []
        self._suspects: dict[tuple, _Suspect] = {}
        self._batcher = _Batcher()
        self._inbox: queue.Queue = queue.Queue()
        self._halt = threading.Event()
        self._worker = threading.Thread(target=self._serve, name="detector-service", daemon=True)
        self._worker.start()

    # ------------------------------------------------------------------ coordinator-facing
    def handle(self, worker_id: str, report: dict) -> None:
        """Called on the coordinator's message path; never blocks."""
        if report.get("kind") == "timing":
            self._inbox.put((worker_id, report))

    def stop(self) -> None:
        self._halt.set()
        self._inbox.put(None)

    def drain(self, timeout: float = 5.0) -> None:
        """Wait until the queued reports are processed (tests)."""
        deadline = time.monotonic() + timeout
        while not self._inbox.empty() and time.monotonic() < deadline:
            time.sleep(0.01)
        time.sleep(0.05)  # the report being processed right now

    def _serve(self) -> None:
        while not self._halt.is_set():
            item = self._inbox.get()
            if item is None:
                return
            try:
                if self.common_mode:
                    for batch in self._batcher.add(*item):
                        self._process_batch(batch)
                else:
                    self._process(*item)
            except Exception:  # noqa: BLE001 -- detection must never take the coordinator down
                log.exception("timing report processing failed")

    # ------------------------------------------------------------------ processing
    @staticmethod
    def _per_layer(report: dict) -> list[tuple[float, float, float]]:
        """Samples as one layer's full work: a rank runs 1 / (tp * cp) of each of its layers."""
        share = max(1, report["tp"]) * max(1, report.get("cp", 1))
        per = share / max(1, report["layers"])
        return [(n, s, sec * per) for n, s, sec in report["samples"]]

    def _expected(self, samples) -> float | None:
        if self.rls.n < self.rls.warmup:
            return None
        return sum(max(self.rls.predict(n, s), 1e-9) for n, s, _ in samples)

    def _process_batch(self, batch: list[tuple[str, dict]]) -> None:
        common = 1.0
        ratios = []
        for _, report in batch:
            samples = self._per_layer(report)
            expected = self._expected(samples) if samples else None
            if expected is not None:
                ratios.append(sum(sec for *_, sec in samples) / expected)
        if len(ratios) >= 3:
            common = max(statistics.median(ratios), 1e-9)
        for worker_id, report in batch:
            self._process(worker_id, report, common)

    def _process(self, worker_id: str, report: dict, common: float = 1.0) -> None:
        devices, gen, it = tuple(report["devices"]), report.get("gen"), report["iteration"]
        samples = [(n, s, sec / common) for n, s, sec in self._per_layer(report)]
        if not samples:
            return
        observed = sum(sec for *_, sec in samples)
        expected = self._expected(samples)
        hit = self.detectors.setdefault((gen, devices), FailSlowDetector(**self.detector_kw)).observe(
            it, observed, expected)
        for sample in samples:
            self.rls.update(*sample)
        if hit is not None and expected is not None:
            self._suspects[devices] = _Suspect(gen, hit.magnitude, it)
            log.warning("fail-slow on %s: %.2fx slower", devices, hit.magnitude)
        suspect = self._suspects.get(devices)
        if suspect is not None and suspect.gen == gen:
            self._decide(devices, suspect, it, observed)

    def _decide(self, devices: tuple, suspect: _Suspect, it: int, observed: float) -> None:
        current, best, cost = self._price(devices, suspect, observed)
        decision = self.policies.setdefault(devices, SkiRentalPolicy(**self.policy_kw)).observe(it, current, best, cost)
        self.events.append(dict(iteration=it, devices=list(devices), ratio=suspect.ratio, act=decision.act,
                                reason=decision.reason, current_s=current, best_s=best, reconfig_s=cost))
        if not decision.act:
            return
        del self._suspects[devices]
        speed = 1.0 / suspect.ratio
        for dev in devices:
            self.speeds[dev] = speed
            self.coord.set_health(dev, p=speed)
        self.coord.request_replan(f"failslow:{','.join(devices)}")

    def _price(self, devices: tuple, suspect: _Suspect, observed: float) -> tuple[float, float, float]:
        if self.what_if is None:
            return observed, observed / suspect.ratio, self.reconfig_cost_s
        if suspect.price is None:
            assumed = {**self.speeds, **{d: 1.0 / suspect.ratio for d in devices}}
            priced = self.what_if(self.coord.payload, assumed)
            suspect.price = (priced.current_s, priced.mitigated_s, priced.reconfig_s)
        return suspect.price
