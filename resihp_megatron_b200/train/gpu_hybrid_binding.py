"""Binding of the GPU hybrid-parallel runtime (TP + SP x PP x DP on the kernels) to the
resilient training loop, so ``resihp-run`` drives GPU training through failures.

Per generation: the coordinator's payload carries the plan and its validated schedule; the
worker builds the TP, DP-set and pipeline-channel groups (``runtime.gpu_runtime.gpu_group_specs``),
a ``GPUHybridRuntime`` for its slot, and moves the committed state into the new layout slice by
slice (``state.transfer_plan`` restricted to up-to-date holders, executed by the transfer engine
over the new communicators, or peer to peer over NVLink on GPUs).  The optimizer state is kept
whole on every replica (``zero=False``) so that the loss of any one rank leaves a holder of every
slice, and the gradients are all-reduced before the loop's REDUCED point: a failure after it
rolls forward (survivors that hold the reduced gradients step locally).  The committed runtime
stays intact until the new generation commits, so a failure during the build restarts from it.
(Reference: ``resihp/train/hetero_binding.py:48-192`` for the CPU model; the reference's GPU
binding is Megatron's, ``resihp/train/megatron_binding.py``.)
"""

from __future__ import annotations

import time

import torch

from ..models.config import GPTConfig
from ..plan.hetero_plan import HeteroParallelPlan
from ..plan.ir import schedule_from_json
from ..runtime.gpu_executor import TokenSource
from ..state.transaction import TransactionManager


def dist_world_size() -> int:
    import torch.distributed as dist

    return dist.get_world_size() if dist.is_initialized() else 1


class GPUHybridBinding:
    def __init__(self, cfg: GPTConfig, client, mgr, *, micro_batch: int = 1, seq_len: int | None = None,
                 device="cuda", tp_impl: str = "collective", lr: float = 3e-4, seed: int = 0, data_seed: int = 1,
                 migrate: str = "auto", hook=None, checkpointer=None, checkpoint_interval: int = 0, fp8=None):
        """``migrate``: ``"p2p"`` (peer copies over NVLink), ``"engine"`` (NCCL / gloo send-receive)
        or ``"auto"`` (p2p on GPUs).  ``checkpointer`` (``state.checkpoint.SliceCheckpointer``):
        every ``checkpoint_interval`` committed iterations each rank writes its slices; a plan
        that asks to restore (no surviving holder of some slice) loads the newest complete one.
        ``fp8``: an ``Fp8Recipe``; the amax histories are the transactions' rollback buffers and
        migrate with their layers."""
        self.cfg, self.client, self.mgr = cfg, client, mgr
        self.micro_batch = micro_batch
        self.S = seq_len or cfg.seq_len
        self.device = torch.device(device)
        self.tp_impl, self.lr, self.seed = tp_impl, lr, seed
        self.tokens = TokenSource(cfg.vocab_size, micro_batch, self.S, seed=data_seed)
        self.migrate = ("p2p" if self.device.type == "cuda" else "engine") if migrate == "auto" else migrate
        self.hook = hook
        self.checkpointer, self.checkpoint_interval = checkpointer, checkpoint_interval
        self.fp8 = fp8
        self.me = client.worker_id
        self.committed = None  # (plan, runtime)
        self.pending = None
        self.last_transfer: dict = {}
        self.last_recovery: dict = {}

    def _plan(self, payload: dict) -> tuple[HeteroParallelPlan, dict]:
        return HeteroParallelPlan.from_json(payload["plan"]), schedule_from_json(payload["schedule"])

    def group_specs(self, world: list[str], payload: dict) -> list:
        from ..runtime.gpu_runtime import gpu_group_specs
        from ..runtime.gpu_state import partition_sizes

        plan, schedule = self._plan(payload)
        return gpu_group_specs(plan, schedule, self.micro_batch * self.S, partition_sizes(self.cfg))

    def _runtime(self, plan, schedule, comms, init: bool):
        from ..runtime.gpu_runtime import GPUHybridRuntime

        return GPUHybridRuntime(self.cfg, plan, schedule, comms, self.mgr, device=self.device,
                                micro_batch=self.micro_batch, seq_len=self.S, tokens=self.tokens,
                                tp_impl=self.tp_impl, dp_impl="collective", seed=self.seed, lr=self.lr, zero=False,
                                init=init, progress=self.client.set_progress, hook=self.hook, fp8=self.fp8)

    def _specs(self):
        from ..runtime.gpu_state import gpu_tensor_specs

        return gpu_tensor_specs(self.cfg, self.fp8.history if self.fp8 is not None else 0)

    def recover(self, comms, payload: dict, txm: TransactionManager) -> None:
        from ..runtime.gpu_state import KINDS, export_state, gpu_layer_of, import_state
        from ..state.layer_registry import device_layout, holdings
        from ..state.transfer_engine import execute_transfers
        from ..state.transfer_plan import plan_transfers

        started = time.monotonic()
        plan, schedule = self._plan(payload)
        rec = payload["recovery"]
        target = rec["target_iteration"]
        old = self.committed
        if old is not None and self.me in rec["local_step"] and txm.has_reduced_grads:
            old[1].apply_step()  # roll forward: the reduced gradients of the interrupted step
            txm.adopt(target)
        elif old is not None:
            old[1].discard_grads()
            txm.discard()
        rt = self._runtime(plan, schedule, comms, init=old is None or target < 0)
        built = time.monotonic()
        prev = payload.get("previous_plan")
        if rec.get("restore"):
            from ..runtime.gpu_state import load_checkpoint_into

            if self.checkpointer is None:
                raise RuntimeError("restore requested but no checkpointer is configured")
            specs = self._specs()
            it = self.checkpointer.latest_complete({k: (sp.global_shape, sp.dim) for k, sp in specs.items()})
            if it is None:
                raise RuntimeError("no complete checkpoint to restore from")
            load_checkpoint_into(rt, self.checkpointer, it, specs)
            txm.adopt(it)
        elif prev is not None and target >= 0:
            specs = self._specs()
            layer_of = gpu_layer_of(self.cfg.layers)
            old_plan = HeteroParallelPlan.from_json(prev)
            old_h, new_h = holdings(old_plan, specs, layer_of), holdings(plan, specs, layer_of)
            valid = set(rec["up_to_date"]) | set(rec["local_step"])
            tplan = plan_transfers(old_h, new_h, valid_sources=valid, node_of=payload.get("nodes", {}))
            if tplan.lost:
                raise RuntimeError(f"{len(tplan.lost)} state slices have no surviving holder")
            mine_valid = old is not None and self.me in valid
            state, layout = export_state(old[1]) if mine_valid else ({k: {} for k in KINDS}, {})
            t0 = time.monotonic()
            new_layout = device_layout(new_h, self.me)
            if self.migrate == "p2p":
                from ..parallel.migration import migrate_p2p
                from ..parallel.symm import exchange_via_group

                new_state = {k: {key: torch.empty(specs[key].local_shape(iv), dtype=torch.float32, device=self.device)
                                 for key, iv in new_layout.items()} for k in KINDS}
                migrate_p2p(tplan, self.me, list(comms.world), specs=specs, old_h=old_h, new_h=new_h, old_state=state,
                            new_state=new_state, kinds=KINDS, device=self.device, exchange=exchange_via_group(None))
            else:
                new_state = execute_transfers(tplan, self.me, comms, self.mgr, specs=specs, old_layout=layout,
                                              old_state=state, new_layout=new_layout, kinds=KINDS,
                                              dtype=torch.float32, device=str(self.device))
            import_state(rt, new_state, step=target + 1)
            txm.adopt(target)
            self.last_transfer = {"transfers": len(tplan.transfers), "reuse": len(tplan.reuse),
                                  "received": sum(1 for t in tplan.transfers if t.dst == self.me),
                                  "seconds": time.monotonic() - t0}
        txm.discard()
        self.pending = (plan, rt)
        # where a recovery's build time goes (the communicators were built just before)
        self.last_recovery = {"comms_s": comms.build_seconds, "comms_phases_s": comms.stats.get("phases_s"),
                              "runtime_build_s": round(built - started, 4),
                              "state_s": round(time.monotonic() - built, 4)}

    def build_runtime(self, comms, payload: dict):
        binding = self

        class _Iteration:
            def run_iteration(self, iteration: int) -> float:
                rt = binding.pending_or_committed()
                loss = float(rt.run_iteration(iteration, step=False).item())  # host synchronisation
                binding.check_collectives(rt)
                return loss

        return _Iteration()

    def check_collectives(self, rt) -> None:
        """After the iteration's host synchronisation: NCCL collectives that a dead peer or an
        abort cut short return as if complete, so the iteration is only REDUCED if no abort came
        and every rank was counted in its last all-reduce (otherwise it is replayed)."""
        from ..comm.comm_manager import CommAborted

        if self.mgr.aborted:
            raise CommAborted("aborted while the iteration's collectives were in flight")
        counted = int(round(float(rt.last_participants.item())))
        if counted != dist_world_size():
            raise CommAborted(f"the iteration's last all-reduce counted {counted} of {dist_world_size()} ranks")

    def pending_or_committed(self):
        return (self.pending or self.committed)[1]

    def on_generation_commit(self) -> None:
        if self.committed is not None and self.pending is not None and self.committed[1] is not self.pending[1]:
            self.committed[1].close()
        self.committed, self.pending = self.pending, None

    def optimizer_step(self) -> None:
        self.committed[1].apply_step()

    def discard_grads(self) -> None:
        self.committed[1].discard_grads()

    def after_commit(self, iteration: int, comms) -> None:
        if self.hook is not None:
            # an injected fault at the iteration boundary fires with no kernel of this worker in flight
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            self.hook(iteration, "boundary")
        if not (self.checkpointer and self.checkpoint_interval and (iteration + 1) % self.checkpoint_interval == 0):
            return
        from ..runtime.gpu_state import checkpoint_slices

        rt = self.committed[1]
        self.checkpointer.save(iteration, self.me, checkpoint_slices(rt, self._specs()),
                               extra={"step_count": rt.step_count}, blocking=True)

    def try_resume(self, txm: TransactionManager) -> None:
        pass

    def buffers(self) -> dict[str, torch.Tensor]:
        """The live fp8 amax histories (snapshotted by each transaction, restored on abort)."""
        current = self.pending or self.committed
        return current[1].buffers() if current is not None else {}
