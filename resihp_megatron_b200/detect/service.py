"""Coordinator-side fail-slow pipeline.

timing reports (one per TP group per iteration: forward-chunk seconds + workload features)
-> per-layer, TP x CP-normalised samples -> one shared gated RLS model -> a residual BOCD per
group -> slowdown ratio for the group's devices -> ski-rental decision -> health ``p = 1/ratio``
+ replan request.  The planner reads ``p`` when it builds the next plan, so mitigation (TP
reshaping, repartition, migration, exclusion) reuses the fail-stop machinery.  With a
``what_if`` pricer the rent is (current plan - replanned plan) and the purchase price is the
estimated migration + rebuild time, so a slowdown the planner cannot mitigate never triggers a
reconfiguration.  (Reference: ``resihp/detect/service.py:30-114``.)

Common-mode correction (``common_mode=True``): the reports of one iteration are processed
together, and when at least three groups report, each group's time is divided by the median
ratio observed / predicted over the groups before it reaches its detector and the shared
predictor.  A slowdown of the whole node (contention, a thermal event, a noisy neighbour) moves
every group alike and cancels; a fail-slow device moves only its group and stands out.
"""

from __future__ import annotations

import queue
import statistics
import threading

from .failslow import FailSlowDetector
from .policy import SkiRentalPolicy
from .predictor import RLSPredictor
from ..utils.log import get_logger

log = get_logger(__name__)


class DetectorService:
    def __init__(self, coordinator, *, warmup: int = 6, threshold: float = 0.9, min_increase: float = 0.25,
                 reconfig_cost_s: float = 0.0, min_gain: float = 0.05, min_dwell: int = 0, token_scale: float = 1e3,
                 what_if=None, common_mode: bool = True, window: int = 8):
        self.coord = coordinator
        # a change is reported while it lies within the last ``window`` iterations: noisy timings
        # may need several post-change samples before the posterior is confident
        self.detector_kw = dict(mode="residual", warmup=warmup, threshold=threshold, min_increase=min_increase,
                                cooldown=warmup, window=window)
        self.rls = RLSPredictor(scales=(token_scale, token_scale ** 2, 1.0), gate=0.3, warmup=32)
        self.detectors: dict[tuple, FailSlowDetector] = {}
        self.policy_kw = dict(min_gain=min_gain, min_dwell=min_dwell)
        self.policies: dict[tuple, SkiRentalPolicy] = {}
        self.reconfig_cost_s = reconfig_cost_s
        self.what_if = what_if
        self.speeds: dict[str, float] = {}
        self.events: list[dict] = []
        self.common_mode = common_mode
        self._pending: dict[tuple, dict[tuple, tuple]] = {}  # (gen, iteration) -> {devices: (worker, report)}
        self._groups: dict[object, set] = {}  # groups seen per generation
        self._suspects: dict[tuple, dict] = {}
        self._q: queue.Queue = queue.Queue()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, name="detector-service", daemon=True)
        self._thread.start()

    def handle(self, worker_id: str, report: dict) -> None:
        """Called on the coordinator's message path; never blocks."""
        if report.get("kind") == "timing":
            self._q.put((worker_id, report))

    def stop(self) -> None:
        self._stop.set()
        self._q.put(None)

    def drain(self, timeout: float = 5.0) -> None:
        """Wait until every queued report has been processed (tests)."""
        import time

        end = time.monotonic() + timeout
        while not self._q.empty() and time.monotonic() < end:
            time.sleep(0.01)
        time.sleep(0.05)  # the report being processed

    def _loop(self) -> None:
        while not self._stop.is_set():
            item = self._q.get()
            if item is None:
                return
            try:
                if self.common_mode:
                    self._collect(*item)
                else:
                    self._process(*item)
            except Exception:  # noqa: BLE001 - detection must never take the coordinator down
                log.exception("timing report processing failed")

    def _collect(self, worker_id: str, rep: dict) -> None:
        """Buffer the reports of an iteration; process one when every group of the generation has
        reported it, or when a group is already two iterations further."""
        gen, it = rep.get("gen"), rep["iteration"]
        devices = tuple(rep["devices"])
        seen = self._groups.setdefault(gen, set())
        seen.add(devices)
        self._pending.setdefault((gen, it), {})[devices] = (worker_id, rep)
        for key in sorted(k for k in self._pending if k[0] == gen):
            batch = self._pending[key]
            if set(batch) >= seen or key[1] <= it - 2:
                del self._pending[key]
                self._process_batch(list(batch.values()))

    def _norm(self, rep: dict) -> list[tuple[float, float, float]]:
        layers = max(1, rep["layers"])
        share = max(1, rep["tp"]) * max(1, rep.get("cp", 1))  # one rank does 1/(tp*cp) of a layer
        return [(n, s, sec * share / layers) for n, s, sec in rep["samples"]]

    def _process_batch(self, batch: list[tuple[str, dict]]) -> None:
        factor = 1.0
        if self.rls.n >= self.rls.warmup:
            ratios = []
            for _, rep in batch:
                norm = self._norm(rep)
                if norm:
                    pred = sum(max(self.rls.predict(n, s), 1e-9) for n, s, _ in norm)
                    ratios.append(sum(sec for *_, sec in norm) / pred)
            if len(ratios) >= 3:
                factor = max(statistics.median(ratios), 1e-9)
        for worker_id, rep in batch:
            self._process(worker_id, rep, factor)

    def _process(self, worker_id: str, rep: dict, common: float = 1.0) -> None:
        devices = tuple(rep["devices"])
        norm = [(n, s, sec / common) for n, s, sec in self._norm(rep)]
        if not norm:
            return
        observed = sum(sec for *_, sec in norm)
        predicted = None
        if self.rls.n >= self.rls.warmup:
            predicted = sum(max(self.rls.predict(n, s), 1e-9) for n, s, _ in norm)
        gen = rep.get("gen")
        det = self.detectors.setdefault((gen, devices), FailSlowDetector(**self.detector_kw))
        hit = det.observe(rep["iteration"], observed, predicted)
        for n, s, sec in norm:
            self.rls.update(n, s, sec)
        if hit is not None and predicted is not None:
            self._suspects[devices] = {"gen": gen, "ratio": hit.magnitude, "since": rep["iteration"], "price": None}
            log.warning("fail-slow on %s: %.2fx slower", devices, hit.magnitude)
        sus = self._suspects.get(devices)
        if sus is None or sus["gen"] != gen:
            return
        current, best, cost = self._price(devices, sus, observed)
        policy = self.policies.setdefault(devices, SkiRentalPolicy(**self.policy_kw))
        d = policy.observe(rep["iteration"], current, best, cost)
        self.events.append({"iteration": rep["iteration"], "devices": list(devices), "ratio": sus["ratio"],
                            "act": d.act, "reason": d.reason, "current_s": current, "best_s": best,
                            "reconfig_s": cost})
        if d.act:
            del self._suspects[devices]
            for dev in devices:
                self.speeds[dev] = 1.0 / sus["ratio"]
                self.coord.set_health(dev, p=1.0 / sus["ratio"])
            self.coord.request_replan(f"failslow:{','.join(devices)}")

    def _price(self, devices: tuple, sus: dict, observed: float) -> tuple[float, float, float]:
        if self.what_if is None:
            return observed, observed / sus["ratio"], self.reconfig_cost_s
        if sus["price"] is None:
            speeds = dict(self.speeds)
            speeds.update({d: 1.0 / sus["ratio"] for d in devices})
            w = self.what_if(self.coord.payload, speeds)
            sus["price"] = (w.current_s, w.mitigated_s, w.reconfig_s)
        return sus["price"]
