"""Worker main: resilient replica-DP training of the float64 GPT decoder on CPU workers.

Benchmark config 1 -- 8 workers on 2 simulated nodes, 8 micro-batches of 2 x 32 tokens, 4
layers, hidden 64, 4 heads, vocab 512, N(0, 0.02) init from seed 0, uniform tokens from seed 1::

    RESIHP_FAULTS="kill@iter=3:target=n0g3:phase=forward" \\
    resihp-run local --nnodes 2 --nproc-per-node 4 \\
        --planner resihp_megatron_b200.train.demo_planners:dp_8mb -- python examples/gpt_dp_demo.py --out /tmp/gpt

The gradients are reduced per micro-batch in global micro-batch order, so every survivor's loss
trajectory is bit for bit that of ``runtime.reference_gpt.train_single_process``, failure or not.
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
from resihp_megatron_b200.runtime.optim import Adam  # noqa: E402
from resihp_megatron_b200.runtime.reference_gpt import GPTRefConfig, GPTRefModel, batch, forward_loss  # noqa: E402
from resihp_megatron_b200.train.dp_binding import DPBinding  # noqa: E402
from resihp_megatron_b200.train.resilient_loop import ResilientTrainer  # noqa: E402


def _gpt_runtime_hooks(cfg: GPTRefConfig) -> dict:
    """How the DP runtime batches, scores and counts tokens for the GPT oracle."""
    return {"batch_fn": lambda it, mb: batch(cfg, it, mb),
            "loss_fn": lambda model, b: forward_loss(cfg, model.params, b[0], b[1]),
            "tokens_fn": lambda it: cfg.tokens_per_iteration}


def main(argv=None) -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--iterations", type=int, default=20)
    parser.add_argument("--lr", type=float, default=1e-3)
    parser.add_argument("--timeout", type=float, default=30.0)
    parser.add_argument("--out", required=True)
    args = parser.parse_args(argv)
    torch.set_num_threads(1)

    cfg = GPTRefConfig()
    model = GPTRefModel(cfg)
    optimizer = Adam(model.params, lr=args.lr, betas=(0.9, 0.95))
    client = WorkerClient(hb_interval=0.1).connect()
    mgr = ResilientCommManager("gloo", timeout_s=args.timeout, validate_timeout_s=args.timeout)
    binding = DPBinding(cfg, None, model, optimizer, mgr, client, injector=get_injector(), timeout=args.timeout,
                        canonical=True, runtime_kwargs=_gpt_runtime_hooks(cfg))
    result = ResilientTrainer(client, mgr, binding).run(args.iterations)

    out, me = Path(args.out), client.worker_id
    out.mkdir(parents=True, exist_ok=True)
    (out / f"{me}.json").write_text(json.dumps(dict(
        worker=me, losses={str(it): loss for it, loss in result.losses.items()}, generations=result.generations,
        reconfigurations=result.reconfigurations, step_count=optimizer.step_count)))
    torch.save({name: p.detach() for name, p in model.params.items()}, out / f"{me}.pt")
    mgr.destroy()
    client.close()
    os._exit(0)  # skip interpreter teardown: helper threads may still hold sockets


if __name__ == "__main__":
    main()
