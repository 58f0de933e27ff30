"""Resilient TP (+SP) x PP x DP training of a Llama-shaped model on the GPU runtime.

The coordinator runs the joint planner (``plan.coordinator_adapter``); each worker runs its slot
of the plan on the package's kernels (``runtime.gpu_runtime``), and when the plan changes (a
failure, a fail-slow eviction, a rejoin) moves parameters and Adam moments slice by slice into
the new layout -- peer to peer over NVLink on GPUs::

    resihp-run local --nnodes 1 --nproc-per-node 8 \\
        --planner resihp_megatron_b200.train.demo_planners:gpu_tp2_pp2_dp2 \\
        -- python examples/gpu_hybrid_demo.py --out /tmp/gpu_hybrid

Each worker writes ``<id>.json`` (losses, generations, layout) under ``--out``.
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
from resihp_megatron_b200.train.demo_planners import GPU_DEMO  # noqa: E402
from resihp_megatron_b200.train.gpu_hybrid_binding import GPUHybridBinding  # noqa: E402
from resihp_megatron_b200.train.resilient_loop import ResilientTrainer  # noqa: E402


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iterations", type=int, default=6)
    ap.add_argument("--lr", type=float, default=1e-2)
    ap.add_argument("--timeout", type=float, default=30.0)
    ap.add_argument("--device", default="cuda", help="cuda (this worker's GPU) or cpu (gloo ranks)")
    ap.add_argument("--tp-impl", default="collective", choices=["fused", "collective"])
    ap.add_argument("--fp8", action="store_true", help="block-scaled fp8 projections with per-layer amax history")
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    torch.set_num_threads(1)
    client = WorkerClient(hb_interval=0.1).connect()
    if args.device == "cuda":
        local = int(os.environ.get("RESIHP_LOCAL_RANK", "0"))
        # an agent that pins each worker to one GPU (CUDA_VISIBLE_DEVICES) leaves it device 0
        torch.cuda.set_device(local if local < torch.cuda.device_count() else 0)
        device, backend = f"cuda:{torch.cuda.current_device()}", "nccl"
    else:
        device, backend = "cpu", "gloo"
    mgr = ResilientCommManager(backend, device=device, timeout_s=args.timeout, validate_timeout_s=args.timeout,
                               subgroup_mode="split" if backend == "nccl" else "local")
    injector = get_injector()
    fp8 = None
    if args.fp8:
        from resihp_megatron_b200.models.fp8_linear import Fp8Recipe

        fp8 = Fp8Recipe()
    binding = GPUHybridBinding(GPU_DEMO, client, mgr, micro_batch=1, seq_len=GPU_DEMO.seq_len, device=device,
                               tp_impl=args.tp_impl, lr=args.lr, hook=injector.on_hook if injector else None, fp8=fp8)
    trainer = ResilientTrainer(client, mgr, binding)
    result = trainer.run(args.iterations)
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    me = client.worker_id
    info = {"worker": me, "losses": {str(k): v for k, v in result.losses.items()}, "generations": result.generations,
            "standby": result.standby, "reconfigurations": result.reconfigurations,
            "last_transfer": binding.last_transfer, "last_recovery": binding.last_recovery,
            "build_steps_s": getattr(trainer, "build_steps_s", None)}
    if binding.committed is not None and not result.standby:
        plan, _ = binding.committed
        g = plan.group_of_device(me)
        info["slot"] = None if g is None else {"replica": g.replica, "stage": g.stage, "tp": g.tp,
                                               "layers": list(g.layers)}
        info["generation"] = plan.generation
        # steps recorded in each layer's amax history (an aborted iteration's entry is rolled back)
        info["amax_steps"] = {k: int((v.abs().sum(0) > 0).sum()) for k, v in binding.buffers().items()}
    (out / f"{me}.json").write_text(json.dumps(info))
    mgr.destroy()
    client.close()
    os._exit(0)


if __name__ == "__main__":
    main()
