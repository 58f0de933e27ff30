"""Synthetic training traces of packed variable-length documents, for detector evaluation.

A trace's iteration time comes from the planner's own pipeline simulator, each micro-batch's
forward costing ``layers * (alpha * N + beta * sum l_i^2)`` with multiplicative noise, an
optional injected slowdown of one (replica, stage) group, and *sticky data regimes*: bursts of
long documents that raise the iteration time for several iterations with no hardware fault --
exactly what fools a detector that watches the raw iteration time.
Parity: ``resihp/detect/synthetic.py:19-170`` (same job model, bursts and evaluation modes).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ..plan.hetero_plan import HeteroParallelPlan, StageGroup
from ..plan.simulator import list_schedule


def _features(docs: list[int]) -> tuple[float, float]:
    lengths = np.asarray(docs, dtype=np.float64)
    return float(lengths.sum()), float(lengths @ lengths)


@dataclass
class SyntheticJob:
    stages: int = 4
    replicas: int = 2
    microbatches: int = 8
    token_budget: int = 32768
    doc_log_mean: float = 6.0
    doc_log_sigma: float = 0.9
    long_doc_prob: float = 0.0
    alpha: float = 3.0e-6
    beta: float = 2.0e-10
    layers_per_stage: int = 8
    bwd_ratio: float = 2.0
    noise: float = 0.015
    p2p_seconds: float = 0.002
    burst_prob: float = 0.04
    burst_len_mean: float = 8.0
    burst_long_doc_prob: float = 0.02

    def plan(self) -> HeteroParallelPlan:
        """One device per (replica, stage), one layer per stage, micro-batches split evenly."""
        keys = [(r, s) for s in range(self.stages) for r in range(self.replicas)]
        groups = tuple(StageGroup(r, s, (f"r{r}s{s}",), (s, s + 1)) for r, s in keys)
        row = tuple(m * self.replicas // self.microbatches for m in range(self.microbatches))
        return HeteroParallelPlan(1, tuple(f"r{r}s{s}" for r, s in keys), self.stages, self.stages, self.replicas,
                                  groups, self.microbatches, (row,) * self.stages)

    def _document(self, rng: np.random.Generator, p_long: float) -> int:
        if rng.random() < p_long:
            return int(rng.integers(self.token_budget // 2, self.token_budget + 1))
        drawn = rng.lognormal(self.doc_log_mean, self.doc_log_sigma)
        return int(min(max(1.0, drawn), self.token_budget))

    def sample_workload(self, rng: np.random.Generator, long_doc_prob: float | None = None) -> list[list[int]]:
        """Document lengths packed into each micro-batch's token budget."""
        p_long = self.long_doc_prob if long_doc_prob is None else long_doc_prob
        batches = []
        for _ in range(self.microbatches):
            docs, room = [], self.token_budget
            while room > 0:
                docs.append(min(self._document(rng, p_long), room))
                room -= docs[-1]
            batches.append(docs)
        return batches

    def chunk_work(self, docs: list[int], alpha: float | None = None, beta: float | None = None) -> float:
        tokens, squares = _features(docs)
        a = self.alpha if alpha is None else alpha
        b = self.beta if beta is None else beta
        return self.layers_per_stage * (a * tokens + b * squares)

    def iteration_time(self, workload: list[list[int]], speeds: dict | None = None, rng=None, alpha=None, beta=None,
                       chunk_fn=None) -> tuple[float, dict]:
        """Makespan and per-group forward chunks ``{(r, s): [(mb, seconds)]}``; ``chunk_fn(docs)``
        replaces the forward cost model (the detectors pass their predictor)."""
        slow = speeds or {}
        price = chunk_fn if chunk_fn is not None else (lambda docs: self.chunk_work(docs, alpha, beta))
        forward = list(map(price, workload))
        noise: dict = {}

        def cost(key, op, mb):
            t = forward[mb] / slow.get(key, 1.0)
            if rng is not None:
                if (key, op, mb) not in noise:
                    noise[(key, op, mb)] = float(rng.normal(1.0, self.noise))
                t *= max(noise[(key, op, mb)], 0.5)
            return t * (1.0 if op == "F" else self.bwd_ratio)

        sim = list_schedule(self.plan(), cost, lambda src, dst, kind: self.p2p_seconds)
        chunks: dict = {}
        for op in (o for o in sim.ops if o.op == "F"):
            chunks.setdefault(op.key, []).append((op.mb, op.end - op.start))
        return sim.makespan, chunks


def _service_view(job: SyntheticJob, trace: list[dict], rls, detector_kw: dict) -> dict:
    """One residual detector per (replica, stage) group on its own forward chunks (localises)."""
    from .failslow import FailSlowDetector

    detectors: dict = {}
    hits_at, groups = [], []
    for rec in trace:
        flagged = []
        for key, items in sorted(rec["chunks"].items()):
            feats = [(*_features(rec["workload"][mb]), sec) for mb, sec in items]
            observed = sum(sec for *_, sec in feats)
            expected = sum(max(rls.predict(n, s), 1e-12) for n, s, _ in feats) if rls.n >= 16 else None
            det = detectors.setdefault(key, FailSlowDetector("residual", **detector_kw))
            if det.observe(rec["iteration"], observed, expected) is not None:
                flagged.append(key)
        if flagged:
            hits_at.append(rec["iteration"])
            groups.append(flagged)
        _learn(rls, rec)
    return {"validations": sum(d.validations for d in detectors.values()), "detections": hits_at,
            "groups": groups, "filtered": 0, "rls": rls}


def _learn(rls, rec: dict) -> None:
    for items in rec["chunks"].values():
        for mb, sec in items:
            rls.update(*_features(rec["workload"][mb]), sec)


def evaluate_detector(job: SyntheticJob, trace: list[dict], mode: str, **detector_kw) -> dict:
    """Run one detector over a trace, its prediction coming from an online gated RLS model fed
    to the simulator.  ``mode == "group"``: the runtime service's per-group view."""
    from .failslow import FailSlowDetector
    from .predictor import RLSPredictor

    rls = RLSPredictor(scales=(float(job.token_budget), float(job.token_budget) ** 2, 1.0))
    if mode == "group":
        return _service_view(job, trace, rls, detector_kw)
    det = FailSlowDetector(mode, **detector_kw)
    hits_at = []
    for rec in trace:
        expected = None
        if rls.n >= 16:
            expected = job.iteration_time(rec["workload"],
                                          chunk_fn=lambda docs: max(rls.predict(*_features(docs)), 0.0))[0]
        if det.observe(rec["iteration"], rec["observed"], expected) is not None:
            hits_at.append(rec["iteration"])
        _learn(rls, rec)
    return {"validations": det.validations, "detections": hits_at, "filtered": det.filtered, "rls": rls}


def generate_trace(job: SyntheticJob, iterations: int, *, seed: int = 0, slow_at: int | None = None,
                   slow_group: tuple[int, int] = (0, 1), factor: float = 2.0) -> list[dict]:
    """``iterations`` records (observed time, workload, chunks, flags); from ``slow_at`` on the
    ``slow_group`` runs ``factor`` times slower."""
    rng = np.random.default_rng(seed)
    records, burst = [], 0
    for it in range(iterations):
        if burst == 0 and rng.random() < job.burst_prob:
            burst = 1 + int(rng.geometric(1.0 / job.burst_len_mean))
        bursting = burst > 0
        workload = job.sample_workload(rng, job.burst_long_doc_prob if bursting else None)
        burst = max(burst - 1, 0)
        slowed = slow_at is not None and it >= slow_at
        seconds, chunks = job.iteration_time(workload, {slow_group: 1.0 / factor} if slowed else {}, rng)
        records.append(dict(iteration=it, observed=seconds, workload=workload, chunks=chunks, slow=slowed,
                            burst=bursting))
    return records
