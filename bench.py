#!/usr/bin/env python3
"""Headline benchmark: Llama-3-8B-shaped pre-training step on N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Config (benchmark config 2 shape): 32 layers, hidden 4096, GQA 32q/8kv heads, SwiGLU FFN
14336, vocab 128256, seq 4096, bf16 compute with fp32 master weights and Adam, random
N(0, 0.02) init, uniform random token ids (synthetic).  Weak scaling: 8 sequences per GPU
per step (global batch 64 at 8 GPUs), micro-batch 1, gradient accumulation over the
rest; for N > 1 data parallel with a sharded optimizer.

Device timing: W untimed warm-up steps, then exactly K steps between a barrier +
``torch.cuda.synchronize()`` on each side, timed with CUDA events on the launching stream;
the slowest rank's time is used.  Every step touches > 100 GB (weights, gradients, optimizer
state), far larger than the 126 MB L2, so no separate L2 flush is needed.  SM clocks and
throttle reasons are sampled with ``nvidia-smi`` during the timed region.

End-to-end number (``e2e``): the same K steps again through the public API
``GPUTrainer.train_step``, which copies each step's ids/labels from pinned host memory to the
device and reads the loss back to the host; timed on the host, max over ranks.

Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import faulthandler
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "tokens/sec/box (device, max over ranks) pre/post reconfig; fault→commit s"
SEQS_PER_GPU = 8
BASELINE_PUBLISHED = None  # no published GPU tokens/s of the reference for this metric


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--seq", type=int, default=None, help="sequence length (default: the model's, 4096 for llama3-8b)")
    ap.add_argument("--seqs-per-gpu", type=int, default=None,
                    help=f"sequences per GPU per step (default {SEQS_PER_GPU}; MoE models: 4 and gpt-1.3b: 32, i.e. "
                         "benchmark config 3's global batch 32 and config 4's 256 at 8 GPUs)")
    ap.add_argument("--micro-batch", type=int, default=None,
                    help="sequences per micro-batch; default 1 on one GPU (the unsharded optimizer state leaves "
                         "room for one), 2 on more (bigger GEMMs, fewer partial waves)")
    ap.add_argument("--layers", type=int, default=None, help="override (testing only; result is marked invalid)")
    ap.add_argument("--reconfig", action="store_true",
                    help="N > 1: after the timed steps evict the last rank (planned, e.g. fail-slow), migrate its "
                         "optimizer state peer to peer, and time the same steps on N-1 GPUs (pre/post tokens/s "
                         "and the eviction-to-commit time)")
    ap.add_argument("--dp-impl", choices=["fused", "nccl"], default="fused",
                    help="N > 1: fused NVLink reduction + Adam + gather kernel, or NCCL reduce-scatter/all-gather")
    ap.add_argument("--cuda-graph", action="store_true",
                    help="one GPU: capture the whole step (every micro-batch and the update) in a CUDA graph after "
                         "the warm-up and replay it")
    ap.add_argument("--parallelism", default="auto",
                    help="'auto' (benchmark config 2's layout where it fits N: tp2pp1dp1 at 2 GPUs, tp2pp2dp1 at 4, "
                         "tp2pp2dp2 at 8; data parallel otherwise), 'dp' (data parallel, ZeRO-1) or 'tp{T}pp{P}dp{D}' "
                         "with T*P*D = N: tensor (+ sequence) x pipeline x data parallelism through the plan-driven "
                         "runtime")
    ap.add_argument("--no-auto-reconfig", action="store_true",
                    help="with --parallelism auto: do not run the live reconfiguration that 'auto' adds when the "
                         "layout has a data-parallel replica (the evicted rank's slices need a surviving holder)")
    ap.add_argument("--ep-impl", choices=["peer", "nccl"], default="peer",
                    help="MoE models: expert dispatch / combine over NVLink peer memory, or NCCL all_to_all")
    ap.add_argument("--tp-impl", choices=["fused", "collective"], default="collective",
                    help="with --parallelism tp..: TP collectives through NCCL (default; measured 1.20x the fused "
                         "kernels on 4 B200s at tp2pp2dp1), or fused into the GEMMs over NVLink peer memory")
    ap.add_argument("--fp8", action="store_true",
                    help="block-scaled fp8 projections (E4M3 forward / E5M2 backward, 1x128 activation and 128x128 "
                         "weight scales, amax history 16; benchmark config 4 with --model gpt-1.3b)")
    ap.add_argument("--failstop", choices=["auto", "on", "off"], default="auto",
                    help="hybrid layouts: after the timed steps and the teardown, run a real fail-stop on the same "
                         "GPUs through the control plane (small demo model, one worker SIGKILLed at a step "
                         "boundary) and report its fault->commit phases; 'auto' runs it at --gpus 2 and 4")
    ap.add_argument("--chaos", choices=["auto", "on", "off"], default="auto",
                    help="after the timed steps, run one real-process kill trial of the CPU chaos harness (8 gloo "
                         "workers, coordinator + 2 agents; fault->commit seconds and its phases) through this arm's "
                         "own code; 'auto' runs it at --gpus 1 only")
    ap.add_argument("--reshard", default=None,
                    help="with --parallelism tp..: after the timed steps change the layout live on the same GPUs "
                         "(e.g. tp2pp1dp4 after tp4pp1dp2: benchmark config 4's TP4 -> TP2), migrating parameters, "
                         "Adam moments and amax histories, and time the same steps again")
    return ap.parse_args()


def fp8_recipe(args):
    if not args.fp8:
        return None
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe

    return Fp8Recipe()


def dtype_of(args) -> str:
    return "fp8 (E4M3 fwd / E5M2 bwd, block-scaled) + bf16" if args.fp8 else "bf16"


def parse_layout(text: str) -> tuple[int, int, int] | None:
    import re

    m = re.fullmatch(r"tp(\d+)pp(\d+)dp(\d+)", text)
    return None if m is None else tuple(int(x) for x in m.groups())


CONFIG2_LAYOUTS = {2: "tp2pp1dp1", 4: "tp2pp2dp1", 8: "tp2pp2dp2"}  # benchmark config 2 scaled to N GPUs


def resolve_auto_layout(args, world: int) -> None:
    """``--parallelism auto``: benchmark config 2's TP2 x PP2 x DP2 (+ SP) layout, scaled down to
    the GPUs present (its global batch, 8 sequences per GPU, scales with them); a live
    reconfiguration (eviction of the last rank) is added when the layout has a data-parallel
    replica to take over the evicted rank's slices."""
    if args.parallelism != "auto":
        return
    from resihp_megatron_b200.models.config import get_config

    dense_llama = not get_config(args.model).is_moe and args.model.startswith("llama")
    args.parallelism = CONFIG2_LAYOUTS.get(world, "dp") if dense_llama else "dp"
    layout = parse_layout(args.parallelism)
    if layout is not None and layout[2] >= 2 and not args.no_auto_reconfig and not args.reshard:
        args.reconfig = True


CHAOS_ITERATIONS = 40
# The reference's chaos trial, preceded by a one-rank build of its communicator manager with the
# defaults its demo worker uses: when that build raises, every worker of the trial fails the same
# way at generation 1, and the error is the reason the trial cannot run.
REFERENCE_CHAOS = """
import json, sys
import torch.distributed as dist
from resihp.comm.comm_manager import ResilientCommManager
from resihp.comm.group_spec import GroupSpec
try:
    store = dist.TCPStore("127.0.0.1", 0, 1, True)
    ResilientCommManager("gloo", timeout_s=10).build(1, ["w0"], "w0", [GroupSpec("tp", (0,), "tp", True)], store=store)
    dist.destroy_process_group()
except Exception as e:
    print("ResilientCommManager('gloo').build raised " + type(e).__name__ + ": " + str(e), file=sys.stderr)
    sys.exit(3)
from resihp.bench import chaos
print(json.dumps(chaos.run_trial("kill", iterations={iterations})), flush=True)
"""


def chaos_trial(impl: str, timeout_s: float = 300.0) -> dict:
    """One SIGKILL trial of the chaos harness of ``impl`` (``ours``: this package's
    ``bench.chaos``; ``reference``: the installed reference's own ``resihp.bench.chaos``, stock
    code, run from ``baseline/_ref``) in a child process; returns its fault->commit time and phases
    or an ``unavailable`` reason.  The workers are CPU-only (gloo) and see no GPU."""
    if impl == "ours":
        path, code = ROOT, (f"from resihp_megatron_b200.bench import chaos; "
                            f"chaos.main(['--fault', 'kill', '--iterations', '{CHAOS_ITERATIONS}'])")
    else:
        path = os.path.join(ROOT, "baseline", "_ref")
        code = REFERENCE_CHAOS.format(iterations=CHAOS_ITERATIONS)
    env = dict(os.environ, PYTHONPATH=path, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        proc = subprocess.run([sys.executable, "-c", code], cwd=path, env=env, capture_output=True, text=True,
                              timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"chaos trial did not finish within {timeout_s:.0f} s"}
    rows = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    if proc.returncode != 0 or not rows:
        tail = [ln for ln in (proc.stderr or "").splitlines() if ln.strip() and not ln.startswith(" ")]
        return {"unavailable": f"chaos trial exited {proc.returncode}: " + (" | ".join(tail[-2:]) or "no output")[:400]}
    res = json.loads(rows[-1])
    if "breakdown" in res:  # this package's result layout
        phases, total, exact = res["breakdown"], res["breakdown"].get("total"), res.get("exact")
    else:  # the reference's
        phases = {k: v for k, v in res.items() if k.endswith("_s")}
        total, exact = res.get("total_s"), res.get("correct")
        if not res.get("recovered", True):
            return {"unavailable": "the reference's chaos trial did not recover", "result": res}
    return {"metric": "fault->commit (SIGKILL of 1 of 8 CPU gloo workers, TP2xPP2xDP2 reference MLP)",
            "value": total, "unit": "s", "higher_is_better": False, "phases_s": phases, "exact": exact,
            "iterations": CHAOS_ITERATIONS}


def failstop_trial(world: int, timeout_s: float = 150.0) -> dict:
    """Fault->commit of a real fail-stop on ``world`` GPUs through the control plane
    (``resihp_megatron_b200.bench.gpu_failstop``: the small demo model at benchmark config 2's
    layout scaled to ``world``; a worker is SIGKILLed at an iteration boundary), run in its own
    process group and bounded in time."""
    import signal

    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    proc = subprocess.Popen([sys.executable, "-m", "resihp_megatron_b200.bench.gpu_failstop", "--gpus", str(world)],
                            cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                            start_new_session=True)
    try:
        stdout, _ = proc.communicate(timeout=timeout_s)
    except subprocess.TimeoutExpired:
        os.killpg(proc.pid, signal.SIGKILL)  # the trial's own process group: its coordinator, agent, workers
        proc.communicate()
        return {"unavailable": f"GPU fail-stop trial did not finish within {timeout_s:.0f} s"}
    rows = [ln for ln in stdout.splitlines() if ln.startswith("{")]
    if proc.returncode != 0 or not rows:
        return {"unavailable": f"GPU fail-stop trial exited {proc.returncode}"}
    res = json.loads(rows[-1])
    victim = res["victim"]
    recovered = res["codes"].get(victim) == -9 and all(c == 0 for w, c in res["codes"].items() if w != victim)
    phases = res.get("phases_s") or {}
    return {"metric": "fault->commit (SIGKILL of 1 GPU worker at a step boundary, control plane, NCCL)",
            "value": phases.get("total"), "unit": "s", "higher_is_better": False, "recovered": recovered,
            "phases_s": phases, "gpus": res["gpus"], "layout": res["layout"], "model": "gpu-demo (4 layers)",
            "iterations_completed": {w: len(v) for w, v in res.get("losses", {}).items()},
            "rebuild_s": next(iter((res.get("rebuild_s") or {}).values()), None)}


def want_failstop(args, world: int) -> bool:
    """``auto``: at the GPU counts where the trial has been run (2 and 4); ``on`` anywhere."""
    return args.failstop == "on" or (args.failstop == "auto" and world in (2, 4))


def want_chaos(args, world: int) -> bool:
    return args.chaos == "on" or (args.chaos == "auto" and world == 1)


def reference_unavailable(args) -> None:
    """The reference's GPU training path is Megatron-Core + Transformer Engine
    (resihp/train/megatron_binding.py); neither is installed nor fetchable offline
    (scripts/setup_megatron.sh clones Megatron-LM from GitHub)."""
    why = None
    try:
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        import resihp  # noqa: F401
        try:
            import megatron.core  # noqa: F401
        except Exception:
            why = ("reference installed in baseline/_ref, but its only GPU training path (MegatronBinding) needs "
                   "Megatron-Core + Transformer Engine, which are not installed and cannot be fetched offline; its "
                   "runnable model is a float64 CPU MLP stack, not this config")
    except Exception as e:  # noqa: BLE001
        why = f"reference not importable from baseline/_ref: {e}"
    if why is None:
        why = "reference Megatron path present but not wired into this bench"
    if int(os.environ.get("RANK", "0")) == 0:
        out = {"impl": "reference", "unavailable": why}
        if want_chaos(args, int(os.environ.get("WORLD_SIZE", "1"))):
            out["chaos"] = chaos_trial("reference")
        print(json.dumps(out), flush=True)


class ClockSampler:
    """Samples SM clocks and throttle reasons of the GPUs in use while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices):
        self.indices = set(indices)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                if int(f[0]) not in self.indices:
                    continue
                mhz.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


def main() -> None:
    faulthandler.enable()
    args = _args()
    if args.impl == "reference":
        reference_unavailable(args)
        return

    import torch
    import torch.distributed as dist

    from resihp_megatron_b200 import ops
    from resihp_megatron_b200.models.config import get_config
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer, init_distributed

    from resihp_megatron_b200.models.config import get_config as _get_config

    if args.seq is None:
        args.seq = _get_config(args.model).seq_len
    if args.seqs_per_gpu is None:  # the benchmark configs' global batches at 8 GPUs: 64, 32 (MoE), 256 (gpt-1.3b)
        args.seqs_per_gpu = {"gpt-1.3b": 32}.get(args.model, 4 if _get_config(args.model).is_moe else SEQS_PER_GPU)
    rank, world, local = init_distributed()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    resolve_auto_layout(args, world)
    if args.parallelism == "ep" or get_config(args.model).is_moe:
        run_moe(args, rank, world, local)
        return
    if args.parallelism != "dp":
        run_hybrid(args, rank, world, local)
        return
    cfg = get_config(args.model, seq_len=args.seq)
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    global_batch = args.seqs_per_gpu * world
    if args.micro_batch is None:
        args.micro_batch = 1 if world == 1 else 2
    group = dist.group.WORLD if world > 1 else None
    trainer = GPUTrainer(cfg, global_batch=global_batch, micro_batch=args.micro_batch, seq_len=args.seq, seed=0,
                         dp_group=group, dp_impl=args.dp_impl, fp8=fp8_recipe(args))
    dev = trainer.device

    # synthetic data: uniform random token ids, next-token labels, one batch per step
    n_batches = args.warmup + args.steps
    g = torch.Generator().manual_seed(1)
    host_batches = []
    for _ in range(min(n_batches, 4)):
        seq = torch.randint(0, cfg.vocab_size, (global_batch, args.seq + 1), generator=g)
        lo, hi = rank * trainer.local_batch, (rank + 1) * trainer.local_batch
        ids = seq[lo:hi, :-1].contiguous().pin_memory()
        lab = seq[lo:hi, 1:].contiguous().pin_memory()
        host_batches.append((ids, lab))
    dev_batches = [(i.to(dev), l.to(dev)) for i, l in host_batches]

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up
    for s in range(args.warmup):
        trainer.step_device(*dev_batches[s % len(dev_batches)])
    torch.cuda.synchronize()
    trainer.check()  # a peer that never reached a barrier ends the run here, not after every step
    if args.cuda_graph:
        if world != 1:
            raise SystemExit("--cuda-graph: one GPU only (the data-parallel step's collectives are not captured)")
        trainer.capture_graphs()

    # ---- device-timed region
    sampler = ClockSampler([local] if world == 1 else range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    l0 = ops.launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    loss = None
    for s in range(args.steps):
        loss = trainer.step_device(*dev_batches[s % len(dev_batches)])
    end.record()
    torch.cuda.synchronize()
    barrier()
    launches = ops.launches() - l0
    clocks = sampler.stop() if sampler else None
    trainer.check()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = trainer.tokens_per_step * args.steps
    value = tokens / (ms_max / 1000.0)
    last_loss = float(loss.item())

    # ---- end-to-end region through the public API (H2D of inputs + D2H of the loss every step)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for s in range(args.steps):
        ids, lab = host_batches[s % len(host_batches)]
        trainer.train_step(ids, lab)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = tokens / float(te.item())
    ids0, lab0 = host_batches[0]
    h2d = ids0.numel() * ids0.element_size() + lab0.numel() * lab0.element_size()

    # ---- optional live reconfiguration: the last rank leaves, state migrates, N-1 GPUs continue
    recfg, alive, post_group = None, True, None
    if args.reconfig and 1 < world < 4:
        recfg = {"skipped": "the spare optimizer bank of a live shrink (sized for N - 1 ranks) does not fit next "
                            "to the 8B model's state on 180 GB below 4 GPUs"}
    elif args.reconfig and world >= 4 and args.dp_impl == "fused":
        survivors = list(range(world - 1))
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        post_group = dist.new_group(survivors)
        alive = trainer.shrink(survivors, post_group)
        torch.cuda.synchronize()
        commit_s = time.perf_counter() - t0
        if alive:
            g2 = torch.Generator().manual_seed(2)
            post_batches = []
            for _ in range(min(n_batches, 4)):
                seq = torch.randint(0, cfg.vocab_size, (global_batch, args.seq + 1), generator=g2)
                lo, hi = trainer.batch_offset, trainer.batch_offset + trainer.local_batch
                post_batches.append((seq[lo:hi, :-1].contiguous().to(dev), seq[lo:hi, 1:].contiguous().to(dev)))
            for s in range(max(2, min(args.warmup, 3))):
                trainer.step_device(*post_batches[s % len(post_batches)])
            torch.cuda.synchronize()
            dist.barrier(group=post_group)
            start.record()
            for s in range(args.steps):
                loss2 = trainer.step_device(*post_batches[s % len(post_batches)])
            end.record()
            torch.cuda.synchronize()
            vals = torch.tensor([start.elapsed_time(end), commit_s], device=dev, dtype=torch.float64)
            dist.all_reduce(vals, op=dist.ReduceOp.MAX, group=post_group)
            post_ms, commit_max = vals.tolist()
            recfg = {"kind": "planned eviction of the last rank; optimizer shards migrated peer to peer over NVLink",
                     "n_gpus_post": world - 1, "post_value": trainer.tokens_per_step * args.steps / (post_ms / 1000),
                     "post_ms_per_step": post_ms / args.steps, "evict_to_commit_s": commit_max,
                     "post_micro_batch": trainer.micro_batch, "post_loss": float(loss2.item()),
                     "phases_s_rank0": getattr(trainer, "last_reconfig", None)}

    if rank == 0:
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": (value / BASELINE_PUBLISHED) if BASELINE_PUBLISHED else None,
            "dtype": dtype_of(args),
            "data": "synthetic (uniform random token ids, random-init N(0,0.02) weights)",
            "config": {
                "model": cfg.name + ("" if not args.layers else f"-{args.layers}L-INVALID"),
                "global_batch": global_batch,
                "seq_len": args.seq,
                "micro_batch": args.micro_batch,
                "parallelism": ("tp1pp1dp1" + ("-cudagraph" if args.cuda_graph else "")) if world == 1
                               else f"dp{world}-zero1-{args.dp_impl}",
                "l2": "inputs larger than L2 (each step touches >100 GB of weights/grads/optimizer state)",
                "params": cfg.num_params(),
                "model_tflops_per_gpu": cfg.flops_per_token(args.seq) * value / world / 1e12,
            },
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": 4 * world},
            "gpu_launches": launches,
            "loss": last_loss,
            "impl": "ours",
        }
        if recfg is not None:
            out["reconfig"] = recfg
        if want_chaos(args, world):
            out["chaos"] = chaos_trial("ours")
        print(json.dumps(out), flush=True)
    if world > 1:
        if post_group is not None:
            if alive:
                dist.barrier(group=post_group)
                trainer.close()  # unmap peer memory before the process group goes away
                dist.barrier(group=post_group)
        else:
            dist.barrier()
            trainer.close()
            dist.barrier()
        dist.destroy_process_group()


def _timed_region(args, trainer, rank: int, world: int, local: int) -> dict:
    """Warm-up, device-timed steps (max over ranks), clocks and the end-to-end steps through
    ``trainer.train_step``; the common part of the MoE and hybrid-parallel runs."""
    import torch
    import torch.distributed as dist

    from resihp_megatron_b200 import ops

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        trainer.step_device()
    torch.cuda.synchronize()
    trainer.check()
    sampler = ClockSampler([local] if world == 1 else range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    l0 = ops.launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    loss = None
    for _ in range(args.steps):
        loss = trainer.step_device()
    end.record()
    torch.cuda.synchronize()
    barrier()
    launches = ops.launches() - l0
    clocks = sampler.stop() if sampler else None
    trainer.check()
    t = torch.tensor([start.elapsed_time(end)], device=trainer.device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = trainer.tokens_per_step * args.steps
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    h2d = 0
    for _ in range(args.steps):
        trainer.train_step()
        h2d += trainer.h2d_bytes_last_step
    torch.cuda.synchronize()
    te = torch.tensor([time.perf_counter() - t0], device=trainer.device, dtype=torch.float64)
    hb = torch.tensor([h2d / args.steps], device=trainer.device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        dist.all_reduce(hb)
    return {"ms": ms_max, "value": tokens / (ms_max / 1000.0), "loss": float(loss.item()), "launches": launches,
            "clocks": clocks, "e2e": tokens / float(te.item()), "h2d": int(hb.item())}


def _json_line(args, cfg, world: int, global_batch: int, mb: int, layout: str, r: dict, extra_config: dict) -> dict:
    return {
        "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms"] / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (r["value"] / BASELINE_PUBLISHED) if BASELINE_PUBLISHED else None, "dtype": dtype_of(args),
        "data": "synthetic (uniform random token ids, random-init N(0,0.02) weights)",
        "config": {"model": cfg.name + ("" if not args.layers else f"-{args.layers}L-INVALID"),
                   "global_batch": global_batch, "seq_len": args.seq, "micro_batch": mb, "parallelism": layout,
                   "l2": "inputs larger than L2 (each step touches > 10 GB of weights/grads/optimizer state per GPU)",
                   "params": cfg.num_params(),
                   "model_tflops_per_gpu": cfg.flops_per_token(args.seq) * r["value"] / world / 1e12, **extra_config},
        "clocks": r["clocks"],
        "e2e": {"value": r["e2e"], "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": 4 * world},
        "gpu_launches": r["launches"], "loss": r["loss"], "impl": "ours",
    }


def _post_steps(args, trainer) -> dict:
    """Warm-up and device-timed steps after a reconfiguration (this rank's time)."""
    import torch
    import torch.distributed as dist

    for _ in range(max(2, min(args.warmup, 3))):
        trainer.step_device()
    torch.cuda.synchronize()
    trainer.check()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    loss = None
    for _ in range(args.steps):
        loss = trainer.step_device()
    end.record()
    torch.cuda.synchronize()
    return {"ms": start.elapsed_time(end), "loss": float(loss.item())}


def run_moe(args, rank: int, world: int, local: int) -> None:
    """Mixtral-shaped MoE step (benchmark config 3): dense weights data parallel, experts expert
    parallel over the same ranks, through ``GPUMoETrainer``."""
    import torch
    import torch.distributed as dist

    from resihp_megatron_b200.models.config import get_config
    from resihp_megatron_b200.train.hybrid_trainer import ensure_process_group
    from resihp_megatron_b200.train.moe_trainer import GPUMoETrainer

    ensure_process_group(torch.device("cuda", local))
    cfg = get_config(args.model, seq_len=args.seq)
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    global_batch = args.seqs_per_gpu * world
    mb = args.micro_batch or 1
    trainer = GPUMoETrainer(cfg, global_batch=global_batch, micro_batch=mb, seq_len=args.seq,
                            ep_impl="peer" if args.ep_impl == "peer" else "collective",
                            dp_impl="fused" if args.dp_impl == "fused" else "collective")
    r = _timed_region(args, trainer, rank, world, local)
    recfg = None
    if args.reconfig and world > 1:
        # fail-slow: the last rank's expert compute is stretched 2x from the host (no GPU setting is
        # touched); every rank times its expert GEMMs, the residual-BOCD monitor flags the slow
        # rank, the planner re-places its experts by speed and their state migrates peer to peer
        trainer.enable_failslow(warmup=6)
        dist.barrier()
        for _ in range(8):  # healthy series for the detector's calibration
            trainer.train_step()
        if rank == world - 1:
            trainer.set_slowdown(2.0)
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        slowed_steps = 0
        while not trainer.failslow_events and slowed_steps < 40:
            trainer.train_step()
            slowed_steps += 1
        detect_s = time.perf_counter() - t0
        event = trainer.failslow_events[0] if trainer.failslow_events else None
        post = _post_steps(args, trainer)  # the slow rank stays slow
        vals = torch.tensor([post["ms"], detect_s], device=trainer.device, dtype=torch.float64)
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        post_ms, detect_max = vals.tolist()
        recfg = {"kind": "fail-slow (last rank's expert compute 2x slower, host-injected), detected by residual BOCD "
                         "on per-rank expert time, experts re-placed by speed, expert state migrated",
                 "detected": event is not None, "slowed_steps_to_replacement": slowed_steps,
                 "slow_to_commit_s": detect_max, "event": event,
                 "post_value": trainer.tokens_per_step * args.steps / (post_ms / 1000),
                 "post_ms_per_step": post_ms / args.steps, "phases_s_rank0": trainer.last_reconfig}
    if rank == 0:
        out = _json_line(args, cfg, world, global_batch, mb, trainer.layout, r,
                         {"experts": cfg.num_experts, "top_k": cfg.top_k})
        if recfg is not None:
            out["reconfig"] = recfg
        if want_chaos(args, world):
            out["chaos"] = chaos_trial("ours")
        print(json.dumps(out), flush=True)
    dist.barrier()
    trainer.close()
    dist.barrier()


def run_hybrid(args, rank: int, world: int, local: int) -> None:
    """TP x PP x DP step through ``GPUHybridTrainer`` (same metric, timing and JSON line)."""
    import torch
    import torch.distributed as dist

    from resihp_megatron_b200.models.config import get_config
    from resihp_megatron_b200.train.hybrid_trainer import GPUHybridTrainer, ensure_process_group

    layout = parse_layout(args.parallelism)
    if layout is None or layout[0] * layout[1] * layout[2] != world:
        raise SystemExit(f"--parallelism {args.parallelism!r} is not tp{{T}}pp{{P}}dp{{D}} with T*P*D = {world}")
    tp, pp, dp = layout
    ensure_process_group(torch.device("cuda", local))
    cfg = get_config(args.model, seq_len=args.seq)
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    global_batch = args.seqs_per_gpu * world
    mb = args.micro_batch or 1
    trainer = GPUHybridTrainer(cfg, tp=tp, pp=pp, dp=dp, global_batch=global_batch, micro_batch=mb,
                               seq_len=args.seq, tp_impl=args.tp_impl,
                               dp_impl="fused" if args.dp_impl == "fused" else "collective", fp8=fp8_recipe(args))
    parts = [b - a for a, b in trainer.plan.layer_partition()]
    r = _timed_region(args, trainer, rank, world, local)
    # optional live reconfiguration: the last rank leaves; the planner re-plans the survivors
    # (TP shrink or eviction of its group, min-max layer repartition) and state migrates slice by slice
    recfg, alive = None, True
    if args.reshard:
        new = parse_layout(args.reshard)
        if new is None or new[0] * new[1] * new[2] != world:
            raise SystemExit(f"--reshard {args.reshard!r} is not tp{{T}}pp{{P}}dp{{D}} with T*P*D = {world}")
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        trainer.reshard(*new)
        commit_s = time.perf_counter() - t0
        post = _post_steps(args, trainer)
        vals = torch.tensor([post["ms"], commit_s], device=trainer.device, dtype=torch.float64)
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        post_ms, commit_max = vals.tolist()
        recfg = {"kind": f"live reshard {args.parallelism} -> {args.reshard} on the same GPUs (params, Adam moments"
                         " and amax histories migrated slice by slice)",
                 "layout_post": trainer.layout, "post_value": trainer.tokens_per_step * args.steps / (post_ms / 1000),
                 "post_ms_per_step": post_ms / args.steps, "reshard_to_commit_s": commit_max,
                 "post_loss": post["loss"], "phases_s_rank0": trainer.last_reconfig}
    elif args.reconfig and layout[2] < 2:
        recfg = {"skipped": "no data-parallel replica: the evicted rank's tensor-parallel slices would have no "
                            "surviving holder (a fail-stop here restores from a checkpoint)"}
    elif args.reconfig:
        try:
            recfg, alive = _hybrid_reconfig(args, trainer, world)
        except Exception as e:  # noqa: BLE001 -- the pre-reconfiguration line is still reported
            recfg, alive = {"error": f"{type(e).__name__}: {e}"[:400]}, False
    out = None
    if rank == 0:
        out = _json_line(args, cfg, world, global_batch, mb, trainer.layout, r, {"layers_per_stage": parts})
        if recfg is not None:
            out["reconfig"] = recfg
        if want_chaos(args, world):
            out["chaos"] = chaos_trial("ours")
        if not want_failstop(args, world):
            # printed before the teardown: a rank that fails to leave cleanly cannot lose the line
            print(json.dumps(out), flush=True)
    if alive:
        dist.barrier()
        trainer.close()
        dist.barrier()
    if rank == 0 and want_failstop(args, world):
        # after every rank released its collectives: the GPU fail-stop trial runs its own job
        out["failstop"] = failstop_trial(world)
        print(json.dumps(out), flush=True)


def _hybrid_reconfig(args, trainer, world: int):
    """Planned eviction of the last rank; the survivors re-plan (TP shrink or eviction of its
    group, min-max layer repartition), migrate state slice by slice and run timed steps.
    Returns (record, whether this rank is still in the job)."""
    import torch
    import torch.distributed as dist

    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    alive = trainer.reconfigure([world - 1])
    commit_s = time.perf_counter() - t0
    if not alive:
        return None, False
    for _ in range(max(2, min(args.warmup, 3))):
        trainer.step_device()
    torch.cuda.synchronize()
    trainer.check()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        loss2 = trainer.step_device()
    end.record()
    torch.cuda.synchronize()
    vals = torch.tensor([start.elapsed_time(end), commit_s], device=trainer.device, dtype=torch.float64)
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    post_ms, commit_max = vals.tolist()
    return {"kind": "planned eviction of the last rank; re-planned layout, slice-level state migration",
            "n_gpus_post": dist.get_world_size(), "post_value": trainer.tokens_per_step * args.steps / (post_ms / 1000),
            "post_ms_per_step": post_ms / args.steps, "evict_to_commit_s": commit_max,
            "post_loss": float(loss2.item()), "phases_s_rank0": trainer.last_reconfig,
            "layout_post": trainer.layout}, True


if __name__ == "__main__":
    main()
