"""Planner cost-model calibration (``bench/profile_gpu.py``): least squares recovers a known
profile from per-layer timings, a measured TP throughput fixes ``tp_overhead``, and a committed
calibration is found by layer shape."""

import json
import random

import pytest

from resihp_megatron_b200.bench.profile_gpu import SHAPES, fit_profile, tp_samples_from_throughput
from resihp_megatron_b200.plan.model_spec import ModelProfile, ModelSpec


def _samples(alpha, beta, bwd_ratio, noise=0.0, seed=0):
    rng = random.Random(seed)
    out = []
    for mb, seq in SHAPES:
        tokens, sum_sq = mb * seq, mb * seq * seq
        fwd = (alpha * tokens + beta * sum_sq) * (1 + noise * rng.uniform(-1, 1))
        out.append({"tokens": tokens, "sum_sq": sum_sq, "fwd_s": fwd, "bwd_s": fwd * bwd_ratio})
    return out


def test_fit_recovers_alpha_beta_and_backward_ratio():
    alpha, beta = 3.3e-7, 1.1e-11
    prof = fit_profile(_samples(alpha, beta, 2.3))
    assert prof.alpha == pytest.approx(alpha, rel=1e-6)
    assert prof.beta == pytest.approx(beta, rel=1e-6)
    assert prof.bwd_ratio == pytest.approx(2.3)


def test_fit_is_stable_under_timing_noise():
    alpha, beta = 3.3e-7, 1.1e-11
    prof = fit_profile(_samples(alpha, beta, 2.0, noise=0.02, seed=3))
    assert prof.alpha == pytest.approx(alpha, rel=0.1)
    assert prof.beta == pytest.approx(beta, rel=0.25)


def test_tp_throughput_sets_the_overhead():
    # 2 GPUs at TP2 reach 1.6x one GPU's tokens/s: 1 / (1 + o) = 1.6 / 2  ->  o = 0.25
    assert tp_samples_from_throughput([(2, 1.6, 1.0)]) == [(2, 1 / 1.6, 1.0)]
    prof = fit_profile(_samples(3e-7, 1e-11, 2.0), [(2, 1.6, 1.0)])
    assert prof.tp_overhead == pytest.approx(0.25)
    assert prof.tp_efficiency(2) == pytest.approx(0.8)


def test_calibrated_profile_is_found_by_layer_shape(tmp_path):
    spec = ModelSpec(num_layers=32, hidden=4096, ffn=14336, num_heads=32, num_kv_heads=8, vocab=128256,
                     seq_len=4096)
    other = ModelSpec(num_layers=24, hidden=2048, ffn=8192, num_heads=16, num_kv_heads=16, vocab=50304,
                      seq_len=2048)
    assert ModelProfile.calibrated(spec, tmp_path) is None
    doc = {"shape": {"hidden": 4096, "ffn": 14336, "heads": 32, "kv_heads": 8},
           "profile": ModelProfile(alpha=1e-7, beta=2e-12, bwd_ratio=2.2, tp_overhead=0.2).to_json()}
    (tmp_path / "llama.json").write_text(json.dumps(doc))
    got = ModelProfile.calibrated(spec, tmp_path)
    assert (got.alpha, got.beta, got.bwd_ratio, got.tp_overhead) == (1e-7, 2e-12, 2.2, 0.2)
    assert got.intra_node_bandwidth == ModelProfile.b200(spec).intra_node_bandwidth  # links stay analytic
    assert ModelProfile.calibrated(other, tmp_path) is None
