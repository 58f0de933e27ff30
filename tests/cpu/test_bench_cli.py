"""ResiBench CLI smoke runs (CPU): detection accuracy, planner ablation, the cluster simulator
end to end, the Megatron log parser and the command-line wiring."""

import json

import pytest

from resihp_megatron_b200.bench import megatron_log, runner


def test_detection_and_planner_ablation(tmp_path):
    runner.main(["--out", str(tmp_path), "detection", "--seeds", "2", "--iterations", "90", "--factors", "2.0"])
    res = json.loads((tmp_path / "detection" / "detection.json").read_text())
    assert res["slow"]["2.0"]["group"]["detected"] == 2 and res["healthy"]["group"] == 0
    runner.main(["--out", str(tmp_path), "planner", "--dps", "2"])
    rows = json.loads((tmp_path / "planner" / "ablation.json").read_text())
    one = next(r for r in rows if r["scenario"] == "1 GPU lost")
    assert one["ResiHP"] >= max(v for k, v in one.items() if k not in ("gpus", "dp", "scenario") and v) - 1e-9


def test_sim_cli_with_a_given_calibration(tmp_path):
    (tmp_path / "sim").mkdir()
    (tmp_path / "sim" / "calibration.json").write_text(json.dumps({"beta": 0.5, "overhead": 1.0}))
    runner.main(["--out", str(tmp_path), "sim", "--scales", "1024", "--days", "2", "--seeds", "1", "--spares", "0"])
    data = json.loads((tmp_path / "sim" / "cluster.json").read_text())
    cell = data["fail-stop + fail-slow, spares=0%"][0]
    assert cell["policies"]["Ideal"]["ettr"] >= cell["policies"]["ResiHP"]["ettr"] >= cell["policies"]["NVRx"]["ettr"]


def test_megatron_log_parser(capsys):
    log = "\n".join([
        " [2026-01-01] iteration        1/     100 | consumed samples: 64 | elapsed time per iteration (ms): 9000.0 "
        "| throughput per GPU (TFLOP/s/GPU): 400.0 | global batch size:    64 | lm loss: 1.100000E+01 |",
        "noise line",
        " [2026-01-01] iteration        2/     100 | elapsed time per iteration (ms): 4000.0 | "
        "throughput per GPU (TFLOP/s/GPU): 700.5 | global batch size:    64 | lm loss: 1.050000E+01 |",
        " [2026-01-01] iteration        3/     100 | elapsed time per iteration (ms): 4100.0 | "
        "throughput per GPU (TFLOP/s/GPU): 690.0 | global batch size:    64 | lm loss: 1.000000E+01 |"])
    recs = megatron_log.parse_log(log)
    assert [r.iteration for r in recs] == [1, 2, 3] and recs[1].tflops_per_gpu == 700.5
    s = megatron_log.summarize(recs, skip_first=1, seq_len=4096)
    assert s["median_iter_time_ms"] == pytest.approx(4050.0) and s["final_loss"] == 10.0
    assert s["tokens_per_s"] == pytest.approx(64 * 4096 / 4.05)


def _bench_module():
    import importlib.util
    import os

    path = os.path.join(os.path.dirname(__file__), "..", "..", "bench.py")
    spec = importlib.util.spec_from_file_location("bench_root", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_bench_chaos_key_of_our_arm_is_an_exact_recovery():
    """The ``chaos`` key of the headline line: one SIGKILL trial through this package's harness
    recovers, reports the fault->commit phases, and the survivors stay bit-exact."""
    bench = _bench_module()
    res = bench.chaos_trial("ours", timeout_s=240)
    assert "unavailable" not in res, res
    assert res["unit"] == "s" and res["higher_is_better"] is False and res["exact"] is True
    phases = res["phases_s"]
    assert set(phases) >= {"detect", "abort", "plan", "build_migrate", "commit", "total"}
    assert 0 < res["value"] == phases["total"] < 30


def test_bench_chaos_key_of_the_reference_arm_names_a_reason_or_a_time():
    import os

    bench = _bench_module()
    if not os.path.isdir(os.path.join(bench.ROOT, "baseline", "_ref", "resihp")):
        pytest.skip("reference not installed under baseline/_ref")
    res = bench.chaos_trial("reference", timeout_s=240)
    assert ("unavailable" in res and res["unavailable"]) or res["value"] > 0
