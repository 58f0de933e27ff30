"""Per-generation rebuild of the resources bound to one communicator layout.

A captured CUDA graph bakes in buffer addresses, communicator handles and the layer set; the
symmetric peer-memory heap of the fused kernels maps the previous generation's peers.  Both must
be released *before* the old generation's communicators go away and re-created *after* the new
generation's runtime exists (before READY), or the new generation would replay stale pointers.
``ResilientTrainer`` drives the hooks:

    teardown()                 before the comm manager replaces generation g
    rebuild(comms, payload)    after the binding built generation g+1's runtime
    after_iteration(i)         after every committed iteration (deferred graph capture)

Teardown is best effort -- hooks are released in reverse registration order and a failure is
logged and returned, never raised, so it cannot block recovery; a failed rebuild raises, which
reports ``build_failed`` and retries the generation.
Parity: ``resihp/runtime/generation_hooks.py:32-162`` (same ordering contract; the reference's
hooks manage Transformer Engine userbuffers and Megatron CUDA graphs, ours the peer-memory heap
and the engine's step graphs).
"""

from __future__ import annotations

from typing import Callable, Protocol

from ..plan.hetero_plan import HeteroParallelPlan
from ..utils.log import get_logger

log = get_logger(__name__)


class GenerationHook(Protocol):
    def teardown(self) -> None: ...
    def rebuild(self, comms, payload: dict) -> None: ...


class GenerationHooks:
    def __init__(self, hooks=()):
        self.hooks = list(hooks)

    def register(self, hook) -> None:
        self.hooks.append(hook)

    def teardown(self) -> list[str]:
        """Release every hook, last registered first; returns the failures as text."""
        failures = []
        for hook in self.hooks[::-1]:
            name = type(hook).__name__
            try:
                hook.teardown()
            except Exception as err:  # noqa: BLE001 -- release is best effort
                log.warning("teardown of %s failed: %s", name, err)
                failures.append(f"{name}: {err}")
        return failures

    def rebuild(self, comms, payload: dict) -> None:
        for hook in self.hooks:
            hook.rebuild(comms, payload)

    def after_iteration(self, iteration: int) -> None:
        for hook in filter(lambda h: hasattr(h, "after_iteration"), self.hooks):
            hook.after_iteration(iteration)


def uniform_contiguous_tp(plan: HeteroParallelPlan) -> int | None:
    """The TP degree if every TP group of the plan is an aligned block of consecutive ranks of one
    common size (what fixed-shape peer buffers assume), else None."""
    degrees = {g.tp for g in plan.stage_groups}
    if len(degrees) != 1:
        return None
    (tp,) = degrees
    blocks = (plan.slice_ranks(g, c) for g in plan.stage_groups for c in range(g.cp))
    aligned = all(b[0] % tp == 0 and list(b) == list(range(b[0], b[0] + tp)) for b in blocks)
    return tp if aligned else None


class SymmetricHeapHook:
    """The per-generation symmetric peer-memory heap of the fused TP / DP / EP kernels.

    ``factory(comms, payload)`` builds the new generation's heap (exchanging handles under the
    generation's store prefix); ``teardown`` closes the old one, which raises its abort word,
    waits for kernels in flight and unmaps the peers.  Any layout the plan names is supported,
    so the hook is disabled only when there is no factory."""

    def __init__(self, factory: Callable[[object, dict], object] | None):
        self.factory = factory
        self.heap = None
        self.rebuilds = 0

    @property
    def enabled(self) -> bool:
        return self.factory is not None

    def teardown(self) -> None:
        heap, self.heap = self.heap, None
        closer = getattr(heap, "close", None)
        if closer is not None:
            closer()

    def rebuild(self, comms, payload: dict) -> None:
        if self.enabled:
            self.heap = self.factory(comms, payload)
            self.rebuilds += 1


class CudaGraphHook:
    """The engine's step graphs are dropped with the old generation and captured again after
    ``warmup`` eager iterations of the new one (the eager steps absorb the allocator's first-use
    growth).  The engine provides ``drop_graphs()`` and ``capture_graphs()``."""

    def __init__(self, engine_fn: Callable[[], object] | None = None, warmup: int = 1):
        self.engine_fn, self.warmup = engine_fn, warmup
        self.eager_left = 0
        self.captures = 0

    def _engine_call(self, method: str) -> None:
        engine = self.engine_fn() if self.engine_fn is not None else None
        fn = getattr(engine, method, None)
        if fn is not None:
            fn()

    def teardown(self) -> None:
        self._engine_call("drop_graphs")

    def rebuild(self, comms, payload: dict) -> None:
        self.eager_left = self.warmup

    def after_iteration(self, iteration: int) -> None:
        if self.eager_left == 0:
            return
        self.eager_left -= 1
        if self.eager_left == 0:
            self._engine_call("capture_graphs")
            self.captures += 1
