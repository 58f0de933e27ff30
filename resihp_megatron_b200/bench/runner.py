"""ResiBench: ``resihp-bench <experiment>`` writes JSON and Markdown under ``--out``.

    resihp-bench detection    fail-slow detection accuracy on synthetic packed-data traces
    resihp-bench planner      planner ablation (TP shrink / repartition / migration / replica drop)
    resihp-bench calibrate    fit the cluster simulator's ResiHP model to the real planner
    resihp-bench sim          trace-driven ETTR at 1K-64K GPUs vs torchft, NVRx, ReCycle, Oobleck, Greyhound
    resihp-bench chaos        real-process chaos on CPU: MTTR breakdown and exactness check
    resihp-bench kernels ...  sm_100a kernel microbenchmarks (GPU), see ``bench.kernels``
    resihp-bench megatron-log FILE [SEQ]   parse a Megatron-LM log of a comparison run
    resihp-bench tp-sweep | moe-sweep | migration-sweep ...   multi-GPU sweeps (under torchrun)
    resihp-bench all          detection, planner, calibrate, sim, chaos

Parity: ``resihp/bench/runner.py:93-137`` (the same experiment names and flags, plus the GPU ones).
"""

from __future__ import annotations

import argparse
import importlib
import json
import time
from pathlib import Path
from typing import Callable

_EXPERIMENTS: dict[str, Callable] = {}
PASS_THROUGH = ("kernels", "megatron-log", "tp-sweep", "moe-sweep", "migration-sweep")
# experiment -> its flags: (name, argparse keyword arguments)
_FLAGS = {
    "detection": [("--seeds", dict(type=int, default=20)), ("--iterations", dict(type=int, default=120)),
                  ("--slow-at", dict(type=int, default=70)), ("--factors", dict(default="1.3,1.6,2.0")),
                  ("--horizon", dict(type=int, default=10))],
    "planner": [("--dps", dict(default="2,4"))],
    "calibrate": [],
    "sim": [("--scales", dict(default="1024,4096,16384,32768,65536")), ("--days", dict(type=float, default=30.0)),
            ("--seeds", dict(type=int, default=5)), ("--spares", dict(default="0,0.02")),
            ("--sensitivity", dict(action="store_true"))],
    "chaos": [("--trials", dict(type=int, default=3)), ("--faults", dict(default="kill,hang,slow"))],
    "all": [("--quick", dict(action="store_true", help="fewer seeds and trials"))],
}


def experiment(name: str):
    def register(fn):
        _EXPERIMENTS[name] = fn
        return fn

    return register


def _publish(folder: Path, stem: str, data, markdown: str) -> None:
    folder.mkdir(parents=True, exist_ok=True)
    (folder / f"{stem}.json").write_text(json.dumps(data, indent=2, default=str))
    (folder / f"{stem}.md").write_text(markdown + "\n")
    print(markdown)


@experiment("detection")
def _detection(args) -> None:
    from . import detection

    factors = [float(x) for x in args.factors.split(",")]
    res = detection.run(args.seeds, args.iterations, args.slow_at, factors, args.horizon)
    _publish(Path(args.out) / "detection", "detection", res, detection.to_markdown(res))


@experiment("planner")
def _planner(args) -> None:
    from . import planner_ablation

    rows = planner_ablation.run(tuple(map(int, args.dps.split(","))))
    _publish(Path(args.out) / "planner", "ablation", rows, planner_ablation.to_markdown(rows))


def _cached_calibration(out: Path) -> dict:
    from ..sim.calibrate import calibrate

    cached = out / "sim" / "calibration.json"
    if not cached.exists():
        cached.parent.mkdir(parents=True, exist_ok=True)
        cached.write_text(json.dumps(calibrate(), indent=2))
    return json.loads(cached.read_text())


@experiment("calibrate")
def _calibrate(args) -> None:
    from ..sim.calibrate import calibrate

    res = calibrate()
    rows = [f"| {dp} | {k} | {v:.3f} | {res['model'][dp][k]:.3f} |"
            for dp, scenario in res["measured"].items() for k, v in scenario.items()]
    md = (f"beta = {res['beta']}, overhead = {res['overhead']}, rmse = {res['rmse']:.4f}\n\n"
          "| DP | scenario | planner | model |\n|---|---|---|---|\n" + "\n".join(rows))
    _publish(Path(args.out) / "sim", "calibration", res, md)


@experiment("sim")
def _sim(args) -> None:
    from ..sim import experiments as ex

    out = Path(args.out)
    calib = _cached_calibration(out)
    scales = tuple(map(int, args.scales.split(",")))
    data, report = {"calibration": calib}, []
    settings = (("fail-stop only", {"slow_per_gpu_day": 0.0}), ("fail-stop + fail-slow", {}))
    for spare in map(float, args.spares.split(",")):
        for label, trace_kw in settings:
            key = f"{label}, spares={spare:.0%}"
            cells = data[key] = [ex.run_cell(g, args.days, args.seeds, calib, trace_kw=trace_kw, spare_frac=spare)
                                 for g in scales]
            focus = next((c for c in cells if c["gpus"] == 16384), cells[-1])
            report += [f"\n### ETTR, {key} ({args.days:.0f} days, {args.seeds} seeds)\n", ex.scale_table(cells),
                       f"\n#### Breakdown at {focus['gpus']:,} GPUs\n", ex.breakdown_table(focus)]
    if args.sensitivity:
        data["sensitivity"] = sens = ex.sensitivity(calib, days=args.days, seeds=max(1, args.seeds // 2))
        report += ["\n### Sensitivity at 16,384 GPUs (fail-stop + fail-slow, no spares)\n", ex.sensitivity_table(sens)]
    _publish(out / "sim", "cluster", data, "\n".join(report))


@experiment("chaos")
def _chaos(args) -> None:
    from . import chaos

    res = chaos.run(args.trials, tuple(args.faults.split(",")))
    _publish(Path(args.out) / "chaos", "chaos", res, chaos.to_markdown(res))


def _pass_through(module: str):
    def run(args) -> None:
        importlib.import_module(f"resihp_megatron_b200.bench.{module}").main(args.rest)

    return run


for _name, _module in (("kernels", "kernels"), ("megatron-log", "megatron_log"), ("tp-sweep", "tp_sweep"),
                       ("moe-sweep", "moe_sweep"), ("migration-sweep", "migration_sweep")):
    # the multi-GPU sweeps run one process per GPU: ``torchrun --nproc-per-node N -m
    # resihp_megatron_b200.bench.runner <sweep> ...``
    experiment(_name)(_pass_through(_module))


@experiment("all")
def _all(args) -> None:
    quick = args.quick
    for sub in (["detection", "--seeds", "10" if quick else "20"], ["planner"], ["calibrate"],
                ["sim", "--seeds", "2" if quick else "5"] + ([] if quick else ["--sensitivity"]),
                ["chaos", "--trials", "1" if quick else "3"]):
        main(["--out", args.out, *sub])


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="resihp-bench", description=__doc__,
                                     formatter_class=argparse.RawTextHelpFormatter)
    parser.add_argument("--out", default="results")
    commands = parser.add_subparsers(dest="cmd", required=True)
    for name, flags in _FLAGS.items():
        sub = commands.add_parser(name)
        for flag, kw in flags:
            sub.add_argument(flag, **kw)
    for name in PASS_THROUGH:
        commands.add_parser(name, add_help=False).add_argument("rest", nargs=argparse.REMAINDER)
    return parser


def main(argv=None) -> None:
    parser = build_parser()
    args, unknown = parser.parse_known_args(argv)
    if unknown:
        if args.cmd not in PASS_THROUGH:
            parser.error(f"unrecognized arguments: {' '.join(unknown)}")
        args.rest = [*unknown, *args.rest]
    started = time.monotonic()
    _EXPERIMENTS[args.cmd](args)
    print(f"[resihp-bench {args.cmd}] {time.monotonic() - started:.1f}s")


if __name__ == "__main__":
    main()
