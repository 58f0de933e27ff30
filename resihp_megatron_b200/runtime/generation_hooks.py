"""Per-generation rebuild of resources bound to one communicator layout.

Captured CUDA graphs bake in buffer addresses, communicator handles and the layer set; the
symmetric peer-memory heap of the fused kernels maps the previous generation's peers.  Both must
be released *before* the old generation's communicators are destroyed and re-created *after*
the new generation's runtime exists (before READY), or the new generation replays stale
pointers.  ``ResilientTrainer`` drives the hooks:

    teardown()                 before ResilientCommManager.build() replaces generation g
    rebuild(comms, payload)    after the binding built generation g+1's runtime
    after_iteration(i)         after every committed iteration (deferred graph capture)

Teardown is best effort (a failed release must not block recovery); a failed rebuild raises,
which reports ``build_failed`` and retries the generation.
(Reference: ``resihp/runtime/generation_hooks.py:32-162``, whose hooks manage Transformer Engine
userbuffers and Megatron CUDA graphs.)
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
        errors = []
        for h in reversed(self.hooks):
            try:
                h.teardown()
            except Exception as e:  # noqa: BLE001
                log.warning("teardown of %s failed: %s", type(h).__name__, e)
                errors.append(f"{type(h).__name__}: {e}")
        return errors

    def rebuild(self, comms, payload: dict) -> None:
        for h in self.hooks:
            h.rebuild(comms, payload)

    def after_iteration(self, iteration: int) -> None:
        for h in self.hooks:
            fn = getattr(h, "after_iteration", None)
            if fn is not None:
                fn(iteration)


def uniform_contiguous_tp(plan: HeteroParallelPlan) -> int | None:
    """The TP degree when every TP group of the plan is an aligned, rank-contiguous block of the
    same size (the layout fixed-shape peer buffers are built for), else ``None``."""
    tps = {g.tp for g in plan.stage_groups}
    if len(tps) != 1:
        return None
    tp = tps.pop()
    for g in plan.stage_groups:
        for i in range(g.cp):
            ranks = plan.slice_ranks(g, i)
            if ranks != tuple(range(ranks[0], ranks[0] + tp)) or ranks[0] % tp:
                return None
    return tp


class SymmetricHeapHook:
    """Per-generation symmetric peer-memory heap of the fused TP/DP/EP kernels.

    ``factory(comms, payload)`` builds the heap for the new generation (exchanging handles over
    the generation's store prefix); ``teardown`` raises the abort word, waits for in-flight
    kernels and unmaps the peers.  Heterogeneous layouts are supported (the heap maps whatever
    groups the plan names), so ``enabled`` is False only without a factory.
    """

    def __init__(self, factory: Callable[[object, dict], object] | None):
        self.factory = factory
        self.heap = None
        self.rebuilds = 0

    @property
    def enabled(self) -> bool:
        return self.factory is not None

    def teardown(self) -> None:
        if self.heap is not None:
            close = getattr(self.heap, "close", None)
            if close is not None:
                close()
            self.heap = None

    def rebuild(self, comms, payload: dict) -> None:
        if self.factory is None:
            return
        self.heap = self.factory(comms, payload)
        self.rebuilds += 1


class CudaGraphHook:
    """Graphs of the engine's step are dropped with the old generation and re-captured after
    ``warmup`` eager iterations of the new one (the warm-up absorbs first-iteration allocator
    growth).  ``engine`` exposes ``drop_graphs()`` and ``capture_graphs()``."""

    def __init__(self, engine_fn: Callable[[], object] | None = None, warmup: int = 1):
        self.engine_fn = engine_fn
        self.warmup = warmup
        self.eager_left = 0
        self.captures = 0

    def teardown(self) -> None:
        eng = self.engine_fn() if self.engine_fn else None
        if eng is not None and hasattr(eng, "drop_graphs"):
            eng.drop_graphs()

    def rebuild(self, comms, payload: dict) -> None:
        self.eager_left = self.warmup

    def after_iteration(self, iteration: int) -> None:
        if self.eager_left <= 0:
            return
        self.eager_left -= 1
        if self.eager_left == 0:
            eng = self.engine_fn() if self.engine_fn else None
            if eng is not None and hasattr(eng, "capture_graphs"):
                eng.capture_graphs()
            self.captures += 1
