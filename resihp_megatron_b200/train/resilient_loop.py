"""The framework-agnostic resilient training loop of one worker.

Per iteration::

    begin txn -> run the iteration (abortable) -> REDUCED -> optimizer step -> COMMIT

On a communication failure or a reconfiguration notice the iteration's transaction is rolled
back (RNG and data cursor included) and the worker joins the next generation::

    wait PREPARE(g) -> generation hooks torn down -> comms(g) built -> state recovered
    (roll-forward, peer copy, snapshot or checkpoint) -> runtime built -> hooks rebuilt
    -> READY(g) -> COMMIT(g)

after which the aborted iteration is replayed with the same global batch.  Survivors never
restart.  Everything model-specific comes from a ``RuntimeBinding``, so the same loop drives
the replica-DP runtime, the heterogeneous hybrid-parallel runtime and the GPU engines.
Parity: ``resihp/train/resilient_loop.py:28-160`` (same sequence and binding protocol).
"""

from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field
from typing import Protocol

from ..comm.comm_manager import CommAborted, CommTimeout, GenerationBuildError, GenerationComms, ResilientCommManager
from ..control.worker_client import JobFinished, ReconfigInterrupted, WorkerClient
from ..runtime.generation_hooks import GenerationHooks
from ..state.transaction import TransactionManager
from ..utils.log import get_logger

log = get_logger(__name__)

# errors after which the worker rejoins at the next generation instead of dying
RECOVERABLE = (CommAborted, CommTimeout, GenerationBuildError, RuntimeError, ReconfigInterrupted)


class Runtime(Protocol):
    def run_iteration(self, iteration: int) -> float: ...


class RuntimeBinding(Protocol):
    def group_specs(self, world: list[str], payload: dict) -> list: ...
    def build_runtime(self, comms: GenerationComms, payload: dict) -> Runtime: ...
    def recover(self, comms: GenerationComms, payload: dict, txm: TransactionManager) -> None: ...
    def optimizer_step(self) -> None: ...
    def discard_grads(self) -> None: ...
    def after_commit(self, iteration: int, comms: GenerationComms) -> None: ...
    def try_resume(self, txm: TransactionManager) -> None: ...


@dataclass
class TrainResult:
    losses: dict[int, float] = field(default_factory=dict)
    generations: list[int] = field(default_factory=list)
    reconfigurations: list[dict] = field(default_factory=list)
    standby: bool = False


class _Join(enum.Enum):
    MEMBER = "member"      # in the committed world, runtime ready
    STANDBY = "standby"    # committed, but not in the world
    RETRY = "retry"        # the generation was superseded or its build failed


class ResilientTrainer:
    def __init__(self, client: WorkerClient, mgr: ResilientCommManager, binding: RuntimeBinding, *,
                 txm: TransactionManager | None = None, prepare_timeout: float = 600.0,
                 hooks: GenerationHooks | None = None):
        self.client, self.mgr, self.binding = client, mgr, binding
        self.txm = txm if txm is not None else TransactionManager()
        self.prepare_timeout = prepare_timeout
        self.hooks = hooks if hooks is not None else GenerationHooks()
        self.comms: GenerationComms | None = None
        self.runtime: Runtime | None = None
        self.result = TrainResult()
        client.add_abort_callback(mgr.abort)  # a notice aborts in-flight communication
        buffers = getattr(binding, "buffers", None)
        if buffers is not None:
            self.txm.track_buffers(buffers)

    def run(self, num_iterations: int) -> TrainResult:
        self.binding.try_resume(self.txm)
        try:
            self._rejoin()
            while True:
                self._train_until(num_iterations)
                verdict = self.client.finish(self.txm.committed_iteration, timeout=self.prepare_timeout)
                if verdict == "shutdown":
                    break
                self._rejoin()  # the others still need this worker (e.g. as a state source)
        except JobFinished:
            pass
        return self.result

    # ------------------------------------------------------------------ iterations
    def _step(self, it: int) -> float:
        """One transactional iteration; raises a RECOVERABLE error when it must be replayed."""
        if self.client.immediate_abort_pending():
            raise CommAborted("reconfiguration announced before the iteration started")
        loss = self.runtime.run_iteration(it)
        self.txm.on_reduced()
        self.txm.on_step_begin()
        self.binding.optimizer_step()
        self.txm.on_commit()
        return loss

    def _publish(self, it: int, loss: float) -> None:
        self.result.losses[it] = loss
        self.client.set_progress(iteration=it, phase="committed", in_collective=False)
        self.client.set_recovery_info(**self.txm.recovery_info())
        self.binding.after_commit(it, self.comms)
        self.hooks.after_iteration(it)

    def _train_until(self, num_iterations: int) -> None:
        while (it := self.txm.committed_iteration + 1) < num_iterations:
            if self.runtime is None:
                self._rejoin()
                continue
            self.txm.begin(it)
            try:
                self._publish(it, self._step(it))
                if self.client.reconfig_pending():
                    self._rejoin()
            except RECOVERABLE as err:
                log.warning("iteration %d interrupted: %s", it, err)
                self.txm.abort()
                self._rejoin()

    # ------------------------------------------------------------------ generations
    def _rejoin(self) -> None:
        started = time.monotonic()
        while True:
            self.client.set_recovery_info(**self.txm.recovery_info())
            prepare = self.client.wait_prepare(timeout=self.prepare_timeout)
            t0 = time.monotonic()
            if self.comms is not None:
                self.hooks.teardown()  # before the old communicators go away
            self._steps_s = {"wait_prepare_s": round(t0 - started, 4), "teardown_s": round(time.monotonic() - t0, 4),
                             "rejoin_at": started}
            outcome = self._enter(prepare)
            if outcome is _Join.MEMBER:
                self._record(prepare, started)
                return
            if outcome is _Join.STANDBY:
                self.result.standby = True
                self.result.generations.append(prepare["gen"])

    def _enter(self, prepare: dict) -> _Join:
        gen, world = prepare["gen"], prepare["world"]
        if self.client.worker_id not in world:
            return self._stand_by(gen)
        try:
            self._build(prepare)
        except RECOVERABLE as err:
            log.warning("generation %d build/recovery failed: %s", gen, err)
            self.hooks.teardown()
            self.client.report("build_failed", gen=gen, suspects=list(getattr(err, "suspects", ())),
                               detail=str(err)[:200])
            self.runtime = None
            return _Join.RETRY
        return _Join.MEMBER

    def _stand_by(self, gen: int) -> _Join:
        self.mgr.destroy()
        self.comms = self.runtime = None
        self.client.send_ready(gen, standby=True)
        try:
            self.client.wait_commit(gen, timeout=self.prepare_timeout)
        except ReconfigInterrupted:
            return _Join.RETRY
        return _Join.STANDBY

    def _build(self, prepare: dict) -> None:
        gen, world, payload = prepare["gen"], prepare["world"], prepare["payload"]
        store = tuple(prepare["store_addr"]) if prepare.get("store_addr") else None
        self.comms = None
        steps = getattr(self, "_steps_s", {})
        t = time.monotonic()
        specs = self.binding.group_specs(world, payload)
        t, steps["group_specs_s"] = time.monotonic(), round(time.monotonic() - t, 4)
        comms = self.mgr.build(gen, world, self.client.worker_id, specs, store_addr=store,
                               store_prefix=prepare["store_prefix"])
        t, steps["comms_s"] = time.monotonic(), round(time.monotonic() - t, 4)
        self.binding.recover(comms, payload, self.txm)
        t, steps["recover_s"] = time.monotonic(), round(time.monotonic() - t, 4)
        self.runtime = self.binding.build_runtime(comms, payload)
        t, steps["build_runtime_s"] = time.monotonic(), round(time.monotonic() - t, 4)
        self.hooks.rebuild(comms, payload)
        steps["hooks_rebuild_s"] = round(time.monotonic() - t, 4)
        steps["ready_at"] = time.monotonic()
        steps.update({k + "_at": v for k, v in getattr(self.client, "arrivals", {}).items() if k.endswith(str(gen))})
        self.build_steps_s = steps  # where this worker's time between PREPARE and READY went
        self.comms = comms
        self.client.send_ready(gen)
        self.client.wait_commit(gen, timeout=self.prepare_timeout)
        committed = getattr(self.binding, "on_generation_commit", None)
        if committed is not None:
            committed()

    def _record(self, prepare: dict, started: float) -> None:
        gen = prepare["gen"]
        self.result.generations.append(gen)
        self.result.standby = False
        self.result.reconfigurations.append(dict(
            generation=gen, world=list(prepare["world"]), seconds=time.monotonic() - started,
            committed_iteration=self.txm.committed_iteration, build_seconds=self.comms.build_seconds,
            path=self.comms.path))
        self.client.set_recovery_info(**self.txm.recovery_info())
