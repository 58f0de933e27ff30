"""Coordinator-side fail-slow pipeline.

timing reports (one per TP group per iteration: forward-chunk seconds + workload features)
-> per-layer, TP x CP-normalised samples -> one shared gated RLS model -> a residual BOCD per
group -> slowdown ratio for the group's devices -> ski-rental decision -> health ``p = 1/ratio``
+ replan request.  The planner reads ``p`` when it builds the next plan, so mitigation (TP
reshaping, repartition, migration, exclusion) reuses the fail-stop machinery.  With a
``what_if`` pricer the rent is (current plan - replanned plan) and the purchase price is the
estimated migration + rebuild time, so a slowdown the planner cannot mitigate never triggers a
reconfiguration.  (Reference: ``resihp/detect/service.py:30-114``.)
"""

from __future__ import annotations

import queue
import threading

from .failslow import FailSlowDetector
from .policy import SkiRentalPolicy
from .predictor import RLSPredictor
from ..utils.log import get_logger

log = get_logger(__name__)


class DetectorService:
    def __init__(self, coordinator, *, warmup: int = 6, threshold: float = 0.9, min_increase: float = 0.25,
                 reconfig_cost_s: float = 0.0, min_gain: float = 0.05, min_dwell: int = 0, token_scale: float = 1e3,
                 what_if=None):
        self.coord = coordinator
        self.detector_kw = dict(mode="residual", warmup=warmup, threshold=threshold, min_increase=min_increase,
                                cooldown=warmup)
        self.rls = RLSPredictor(scales=(token_scale, token_scale ** 2, 1.0), gate=0.3, warmup=32)
        self.detectors: dict[tuple, FailSlowDetector] = {}
        self.policy_kw = dict(min_gain=min_gain, min_dwell=min_dwell)
        self.policies: dict[tuple, SkiRentalPolicy] = {}
        self.reconfig_cost_s = reconfig_cost_s
        self.what_if = what_if
        self.speeds: dict[str, float] = {}
        self.events: list[dict] = []
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

    def _loop(self) -> None:
        while not self._stop.is_set():
            item = self._q.get()
            if item is None:
                return
            try:
                self._process(*item)
            except Exception:  # noqa: BLE001 - detection must never take the coordinator down
                log.exception("timing report processing failed")

    def _process(self, worker_id: str, rep: dict) -> None:
        devices = tuple(rep["devices"])
        layers = max(1, rep["layers"])
        share = max(1, rep["tp"]) * max(1, rep.get("cp", 1))  # one rank does 1/(tp*cp) of a layer
        norm = [(n, s, sec * share / layers) for n, s, sec in rep["samples"]]
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
