"""Detection: RLS predictor, BOCD, fail-slow modes on synthetic traces, localisation, ski rental,
DetectorService with a fake coordinator, validation rounds, and the native NCCL profiler plugin
driven through its v5 ABI with ctypes (no NCCL needed)."""

import ctypes

import numpy as np
import pytest

from resihp_megatron_b200.detect.bocd import BOCD
from resihp_megatron_b200.detect.failslow import localize
from resihp_megatron_b200.detect.policy import SkiRentalPolicy
from resihp_megatron_b200.detect.predictor import RLSPredictor, fit_least_squares
from resihp_megatron_b200.detect.service import DetectorService
from resihp_megatron_b200.detect.synthetic import SyntheticJob, evaluate_detector, generate_trace
from resihp_megatron_b200.detect.validation import edge_rounds, ring_edges


def test_rls_learns_and_gates():
    rng = np.random.default_rng(0)
    rls = RLSPredictor(scales=(1e4, 1e8, 1.0))
    for _ in range(200):
        n, s = rng.uniform(1e3, 3e4), rng.uniform(1e6, 5e8)
        rls.update(n, s, 3e-6 * n + 2e-10 * s + 1e-3)
    a, b, c = rls.coefficients()
    assert a == pytest.approx(3e-6, rel=0.05) and b == pytest.approx(2e-10, rel=0.1)
    before = rls.theta.copy()
    assert rls.update(2e4, 1e8, 10 * (3e-6 * 2e4 + 2e-10 * 1e8 + 1e-3)) is False  # a 10x outlier is not learned
    assert np.array_equal(before, rls.theta) and rls.rejected == 1
    samples = [(n, s, 2e-6 * n + 1e-10 * s + 5e-4) for n, s in rng.uniform(1, 1e4, (50, 2))]
    fa, fb, fc = fit_least_squares(samples)
    assert fa == pytest.approx(2e-6, rel=1e-6)


def test_bocd_detects_a_level_shift():
    rng = np.random.default_rng(1)
    b = BOCD(hazard=1 / 100, alpha0=10.0, sigma0=0.05)  # calibrated noise prior, as the detector uses
    xs = list(rng.normal(0, 0.05, 60)) + list(rng.normal(0.7, 0.05, 10))
    probs = []
    for x in xs:
        b.update(x)
        probs.append(b.prob_recent_change(3))
    assert max(probs[10:55]) < 0.5 and max(probs[60:65]) > 0.9  # the first few points are young runs
    assert b.map_run_length() == 10  # ten observations since the shift


def test_residual_detector_ignores_workload_bursts_but_catches_slowdown():
    job = SyntheticJob(burst_prob=0.08, burst_long_doc_prob=0.05)
    healthy = generate_trace(job, 120, seed=3)
    slow = generate_trace(job, 120, seed=3, slow_at=80, factor=2.0)
    g = evaluate_detector(job, healthy, "greyhound")
    r = evaluate_detector(job, healthy, "residual")
    assert r["validations"] <= g["validations"]
    hit = evaluate_detector(job, slow, "group")
    assert hit["detections"] and hit["detections"][0] >= 80
    assert (0, 1) in hit["groups"][0]


def test_localize_and_ski_rental():
    rls = RLSPredictor(scales=(1.0, 1.0, 1.0), warmup=0)
    for n in range(1, 50):
        rls.update(float(n), 0.0, 2.0 * n, force=True)
    p = localize({"g0": [(10.0, 0.0, 20.0)], "g1": [(10.0, 0.0, 40.0)]}, rls)
    assert set(p) == {"g1"} and p["g1"] == pytest.approx(0.5, rel=0.05)
    pol = SkiRentalPolicy(min_gain=0.05, min_dwell=0)
    assert not pol.observe(0, 1.02, 1.0, 5.0).act
    acts = [pol.observe(i, 2.0, 1.0, 3.0).act for i in range(1, 6)]
    assert acts == [False, False, True, False, False]


class FakeCoord:
    def __init__(self):
        self.health = {}
        self.replans = []
        self.payload = None

    def set_health(self, w, **h):
        self.health.setdefault(w, {}).update(h)

    def request_replan(self, reason):
        self.replans.append(reason)


def test_detector_service_flags_a_slow_group():
    coord = FakeCoord()
    svc = DetectorService(coord, warmup=6, reconfig_cost_s=0.0, min_gain=0.05, token_scale=1e3)
    rng = np.random.default_rng(5)
    for it in range(80):
        for g, devs in enumerate((["a0", "a1"], ["b0", "b1"])):
            samples = []
            for _ in range(4):
                n = float(rng.integers(500, 2000))
                s = float(n * rng.integers(50, 400))
                sec = (2e-6 * n + 1e-9 * s) * 4 * (1.0 + rng.normal(0, 0.01))
                if g == 1 and it >= 60:
                    sec *= 2.0
                samples.append((n, s, sec))
            svc.handle("w", {"kind": "timing", "iteration": it, "gen": 1, "devices": devs, "layers": 4, "tp": 2,
                             "cp": 1, "samples": samples})
    svc.drain()
    svc.stop()
    assert coord.replans and coord.replans[0].startswith("failslow:b0,b1")
    assert 0.3 < coord.health["b0"]["p"] < 0.9  # estimated at first detection, before the full window is slow
    assert "a0" not in coord.health


def test_edge_colouring_rounds():
    assert len(edge_rounds(ring_edges(list(range(8))))) == 2
    assert len(edge_rounds(ring_edges(list(range(7))))) == 3
    rounds = edge_rounds(ring_edges(list(range(6))))
    for rnd in rounds:
        ends = [x for e in rnd for x in e]
        assert len(ends) == len(set(ends))


# ------------------------------------------------------------------ native NCCL profiler plugin
class _Coll(ctypes.Structure):
    _fields_ = [("seqNumber", ctypes.c_uint64), ("func", ctypes.c_char_p), ("sendBuff", ctypes.c_void_p),
                ("recvBuff", ctypes.c_void_p), ("count", ctypes.c_size_t), ("root", ctypes.c_int),
                ("datatype", ctypes.c_char_p), ("nChannels", ctypes.c_uint8), ("nWarps", ctypes.c_uint8),
                ("algo", ctypes.c_char_p), ("proto", ctypes.c_char_p), ("parentGroup", ctypes.c_void_p)]


class _P2p(ctypes.Structure):
    _fields_ = [("func", ctypes.c_char_p), ("buff", ctypes.c_void_p), ("datatype", ctypes.c_char_p),
                ("count", ctypes.c_size_t), ("peer", ctypes.c_int), ("nChannels", ctypes.c_uint8),
                ("parentGroup", ctypes.c_void_p)]


class _U(ctypes.Union):
    _fields_ = [("coll", _Coll), ("p2p", _P2p)]


class _Descr(ctypes.Structure):
    _anonymous_ = ("u",)
    _fields_ = [("type", ctypes.c_uint64), ("parentObj", ctypes.c_void_p), ("rank", ctypes.c_int), ("u", _U)]


_INIT = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.c_uint64, ctypes.POINTER(ctypes.c_int),
                         ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p)
_START = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(_Descr))
_STOP = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)
_STATE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p)
_FIN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)


class _Profiler(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("init", _INIT), ("startEvent", _START), ("stopEvent", _STOP),
                ("recordEventState", _STATE), ("finalize", _FIN)]


def test_nccl_profiler_plugin_records_coll_and_p2p(tmp_path, monkeypatch):
    from resihp_megatron_b200.detect.nccl_profile_reader import COLL, P2P, RingReader, find_rings
    from resihp_megatron_b200.detect.nccl_profiler import build

    lib = build(tmp_path / "libresihp_nccl_profiler.so")
    monkeypatch.setenv("RESIHP_NCCL_PROF_DIR", str(tmp_path))
    prof = _Profiler.in_dll(ctypes.CDLL(str(lib)), "ncclProfiler_v5")
    assert prof.name == b"resihp"
    ctx, mask = ctypes.c_void_p(), ctypes.c_int(0)
    assert prof.init(ctypes.byref(ctx), 0xABC, ctypes.byref(mask), b"tp", 1, 4, 2, None) == 0
    assert mask.value == COLL | P2P
    reader = RingReader(find_rings(tmp_path)[0])
    h = ctypes.c_void_p()
    d = _Descr(type=COLL, rank=2)
    d.coll.func, d.coll.count = b"AllReduce", 1024
    prof.startEvent(ctx, ctypes.byref(h), ctypes.byref(d))
    prof.stopEvent(h)
    d2 = _Descr(type=P2P, rank=2)
    d2.p2p.func, d2.p2p.count, d2.p2p.peer = b"Send", 77, 3
    prof.startEvent(ctx, ctypes.byref(h), ctypes.byref(d2))
    prof.stopEvent(h)
    prof.startEvent(ctx, ctypes.byref(h), ctypes.byref(_Descr(type=1 << 3, rank=2)))
    assert h.value is None  # proxy events are not profiled
    recs = reader.poll()
    assert [(r.func, r.count, r.peer, r.type, r.comm_id, r.rank, r.nranks) for r in recs] == [
        ("AllReduce", 1024, -1, COLL, 0xABC, 2, 4), ("Send", 77, 3, P2P, 0xABC, 2, 4)]
    assert all(r.end_ns >= r.start_ns for r in recs) and reader.poll() == []
    reader.close()
    assert prof.finalize(ctx) == 0


def test_common_mode_noise_is_cancelled_and_the_slow_group_still_found():
    """Four groups; iterations 20-29 slow every group 2.5x (node-wide contention: nobody is
    flagged), group 3 alone runs 2x slower from iteration 60 (flagged)."""
    coord = FakeCoord()
    svc = DetectorService(coord, warmup=6, reconfig_cost_s=0.0, min_gain=0.05, token_scale=1e3)
    rng = np.random.default_rng(7)
    groups = [[f"g{g}a", f"g{g}b"] for g in range(4)]
    for it in range(90):
        for g, devs in enumerate(groups):
            samples = []
            for _ in range(4):
                n = float(rng.integers(500, 2000))
                s = float(n * rng.integers(50, 400))
                sec = (2e-6 * n + 1e-9 * s) * 4 * (1.0 + rng.normal(0, 0.01))
                if 20 <= it < 30:
                    sec *= 2.5
                if g == 3 and it >= 60:
                    sec *= 2.0
                samples.append((n, s, sec))
            svc.handle("w", {"kind": "timing", "iteration": it, "gen": 1, "devices": devs, "layers": 4, "tp": 2,
                             "cp": 1, "samples": samples})
    svc.drain()
    svc.stop()
    assert coord.replans and all(r.startswith("failslow:g3a,g3b") for r in coord.replans), coord.replans
    assert all(e["iteration"] >= 60 for e in svc.events)


def test_a_change_that_needs_several_samples_to_be_sure_of_is_still_reported():
    """Residuals recorded from a CPU job whose rank went 2x slow at sample 18: the first
    post-change samples are ambiguous, so the posterior only becomes confident a few samples
    later; the detector must still report the change (a 3-sample window missed it)."""
    import math

    from resihp_megatron_b200.detect.failslow import FailSlowDetector

    xs = [-0.03, 0.34, -0.08, -0.01, -0.22, 0.09, -0.05, -0.25, 0.16, -0.24, -0.03, 0.07, -0.22, 0.02, 0.32, -0.03,
          -0.04, 0.14, 0.48, 0.74, 0.63, 0.42, 0.61, 0.76, 0.49, 0.53, 0.67, 0.25, 0.86, 0.38, 0.62, 0.37, 0.72, 0.55]
    d = FailSlowDetector("residual", warmup=6, threshold=0.9, min_increase=0.5, cooldown=6, window=8)
    hits = [i for i, x in enumerate(xs) if d.observe(i, math.exp(x), 1.0)]
    assert hits and 18 <= hits[0] <= 24, hits


def test_expert_slow_monitor_flags_only_the_slow_rank():
    """Per-row expert times of 8 ranks with 3 % jitter and uneven routing (some ranks get no rows
    in some steps): rank 5 slows 2x at step 20 and is the only one flagged, with a speed near 0.5."""
    import random

    from resihp_megatron_b200.train.moe_failslow import ExpertSlowMonitor

    rng = random.Random(3)
    mon = ExpertSlowMonitor(8, warmup=8)
    flagged = []
    for it in range(40):
        rows = [0 if rng.random() < 0.1 else rng.randint(200, 900) for _ in range(8)]
        times = [n * 0.01 * (1 + 0.03 * (2 * rng.random() - 1)) * (2.0 if r == 5 and it >= 20 else 1.0)
                 for r, n in enumerate(rows)]
        out = mon.observe(it, times, rows)
        if out:
            flagged.append((it, out))
            mon.reset()
    assert flagged, "the slow rank was not detected"
    it, speeds = flagged[0]
    assert 20 <= it <= 26 and set(speeds) == {5} and 0.4 < speeds[5] < 0.6, flagged
    assert all(set(s) == {5} for _, s in flagged)
