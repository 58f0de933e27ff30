"""The zero-bubble B / W split behind the IR's ``W`` instruction.

B produces only the input gradient, which unblocks the previous stage; W later produces the
same micro-batch's weight gradients and fills pipeline bubbles.

* ``AutogradWeightGradStore`` works with any PyTorch module: B differentiates the stage output
  with respect to the stage input (graph retained), W with respect to the parameters.  It is
  the semantic reference of the split.
* ``KernelWeightGradStore`` serves an engine whose backward is already two explicit passes
  (dgrad GEMMs, then wgrad GEMMs): B runs the first, W pops the matching deferred second pass,
  first in first out per model chunk -- and checks that order.
Parity: ``resihp/runtime/weight_grad_store.py:25-84`` (same B/W contract; the reference's GPU
half drives Transformer Engine's delayed wgrad queues).
"""

from __future__ import annotations

import contextlib
from collections import deque
from typing import Callable

import torch


def _accumulate(params: list[torch.Tensor], grads) -> None:
    with torch.no_grad():
        for p, g in zip(params, grads):
            if g is not None:
                p.grad = g if p.grad is None else p.grad.add_(g)


class AutogradWeightGradStore:
    def __init__(self, params: Callable[[], list[torch.Tensor]]):
        self.params = params
        self._deferred: dict = {}  # key -> (output, upstream gradient) whose W has not run

    def backward_input(self, mb, out: torch.Tensor, grad: torch.Tensor | None, inp: torch.Tensor | None):
        """B: the input gradient (None at the first stage); the graph stays alive for W."""
        self._deferred[mb] = (out, grad)
        if inp is None:
            return None
        return torch.autograd.grad(out, inp, grad_outputs=grad, retain_graph=True)[0]

    def compute(self, mb) -> None:
        """W: accumulate the deferred micro-batch's parameter gradients."""
        out, grad = self._deferred.pop(mb)
        trainable = list(filter(lambda p: p.requires_grad, self.params()))
        _accumulate(trainable, torch.autograd.grad(out, trainable, grad_outputs=grad, allow_unused=True))

    def pending(self) -> list:
        return sorted(self._deferred)

    def clear(self) -> None:
        self._deferred.clear()


class KernelWeightGradStore:
    """Deferred weight-gradient passes per model chunk, keyed ``(stage, mb)``, FIFO per chunk."""

    def __init__(self, chunks: dict[int, object]):
        self.chunks = chunks
        self._fifo: dict[int, deque] = {stage: deque() for stage in chunks}

    @contextlib.contextmanager
    def deferring(self, key: tuple[int, int]):
        """Around a B pass: afterwards, queue the chunk's pending wgrad closure for W."""
        yield
        stage, mb = key
        take = getattr(self.chunks[stage], "pop_wgrad", None)
        self._fifo[stage].append((mb, take() if take is not None else (lambda: None)))

    def defer(self, key: tuple[int, int], fn: Callable[[], None]) -> None:
        self._fifo[key[0]].append((key[1], fn))

    def compute(self, key: tuple[int, int]) -> None:
        stage, mb = key
        queue = self._fifo[stage]
        if not queue or queue[0][0] != mb:
            raise RuntimeError(f"W({mb}) of stage {stage} out of B order {[m for m, _ in queue]}: "
                               "wgrad queues are FIFO")
        queue.popleft()[1]()

    def pending(self) -> list[tuple[int, int]]:
        return [(stage, mb) for stage, queue in self._fifo.items() for mb, _ in queue]

    def clear(self) -> None:
        for queue in self._fifo.values():
            queue.clear()
