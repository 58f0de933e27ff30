"""Worker main: dynamic hybrid parallelism with live state migration on the float64 reference
model (CPU ranks, or one GPU per rank).

The coordinator runs the joint TP -> PP -> DP planner (``plan.coordinator_adapter``); each
worker trains its slice of the reference model with heterogeneous TP, uneven PP and stage-level
micro-batch migration, and moves parameters plus Adam state slice by slice whenever the plan
changes::

    resihp-run local --nnodes 2 --nproc-per-node 4 \\
        --planner resihp_megatron_b200.train.demo_planners:hetero_tp2_pp2_dp2 \\
        -- python examples/hetero_demo.py --out /tmp/hetero

``--backend gloo`` runs on the CPU; ``--backend nccl`` puts the same model and instruction streams
on this worker's GPU.  Parameters and batches come from counter-based seeds, so both backends train
the identical model.  Each worker writes ``<id>.json`` (losses, generations, last transfer) and
``<id>.pt`` (its final shards) under ``--out``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402

from resihp_megatron_b200.comm.comm_manager import ResilientCommManager  # noqa: E402
from resihp_megatron_b200.control.worker_client import WorkerClient  # noqa: E402
from resihp_megatron_b200.inject.faults import get_injector  # noqa: E402
from resihp_megatron_b200.runtime.reference_model import RefModelConfig  # noqa: E402
from resihp_megatron_b200.state.rng_data import IndexAddressableSampler  # noqa: E402
from resihp_megatron_b200.train.hetero_binding import HeteroBinding  # noqa: E402
from resihp_megatron_b200.train.resilient_loop import ResilientTrainer  # noqa: E402

OPTIONS = [("--iterations", dict(type=int, default=6)), ("--gbs", dict(type=int, default=16)),
           ("--mbs", dict(type=int, default=2)), ("--lr", dict(type=float, default=1e-2)),
           ("--timeout", dict(type=float, default=30.0)),
           ("--channels", dict(action="store_true", help="dedicated 2-rank groups per pipeline direction")),
           ("--iter-sleep", dict(type=float, default=0.0, help="stretch iterations (demos and chaos runs)")),
           ("--amax-history", dict(type=int, default=0, help="fp8-style delayed-scaling history length")),
           ("--backend", dict(default="gloo", choices=["gloo", "nccl"])), ("--out", dict(required=True))]


def _device(backend: str) -> str:
    if backend != "nccl":
        return "cpu"
    torch.cuda.set_device(int(os.environ.get("RESIHP_LOCAL_RANK", "0")))
    return f"cuda:{torch.cuda.current_device()}"


def _write_result(out: Path, me: str, result, binding: HeteroBinding) -> None:
    out.mkdir(parents=True, exist_ok=True)
    report = dict(worker=me, losses={str(it): loss for it, loss in result.losses.items()},
                  generations=result.generations, standby=result.standby, reconfigurations=result.reconfigurations,
                  last_transfer=binding.last_transfer)
    gen = binding.committed
    if gen is not None and not result.standby:
        report["layout"] = {key: list(span) for key, span in gen.layout.items()}
        report["generation"] = gen.plan.generation
        shards = {k: v.detach().cpu() for k, v in gen.module.named_state().items()}
        shards |= {k: v.cpu() for k, v in gen.module.named_buffer_state().items()}
        torch.save(shards, out / f"{me}.pt")
    (out / f"{me}.json").write_text(json.dumps(report))


def main(argv=None) -> None:
    parser = argparse.ArgumentParser()
    for flag, kw in OPTIONS:
        parser.add_argument(flag, **kw)
    args = parser.parse_args(argv)
    torch.set_num_threads(1)
    client = WorkerClient(hb_interval=0.1).connect()
    device = _device(args.backend)
    mgr = ResilientCommManager(args.backend, device=device, timeout_s=args.timeout, validate_timeout_s=args.timeout)
    binding = HeteroBinding(RefModelConfig(amax_history=args.amax_history, device=device),
                            IndexAddressableSampler(256, args.gbs, args.mbs, seed=7), mgr, client, lr=args.lr,
                            use_channels=args.channels, injector=get_injector(), timeout=args.timeout, chunk=4,
                            iter_sleep=args.iter_sleep)
    result = ResilientTrainer(client, mgr, binding).run(args.iterations)
    _write_result(Path(args.out), client.worker_id, result, binding)
    mgr.destroy()
    client.close()
    os._exit(0)  # skip interpreter teardown: helper threads may still hold sockets


if __name__ == "__main__":
    main()
