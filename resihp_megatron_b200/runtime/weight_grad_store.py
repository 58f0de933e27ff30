"""Zero-bubble B/W split for the IR's ``W`` instruction.

B produces only the input gradient (unblocking the previous stage); W later produces the
weight gradients of the same micro-batch and fills pipeline bubbles.

* ``AutogradWeightGradStore``: any PyTorch module -- B runs ``autograd.grad`` w.r.t. the stage
  input with the graph retained, W runs it w.r.t. the parameters (the semantic reference).
* ``KernelWeightGradStore``: the GPU model's explicit backward is already split into a dgrad
  pass and a wgrad pass (``models/gpt.py``); B runs the dgrad GEMMs, W the queued wgrad GEMMs,
  FIFO per model chunk (checked).
(Reference: ``resihp/runtime/weight_grad_store.py:25-84``, whose GPU half drives Transformer
Engine's delayed wgrad queues.)
"""

from __future__ import annotations

import contextlib
from typing import Callable

import torch


class AutogradWeightGradStore:
    def __init__(self, params: Callable[[], list[torch.Tensor]]):
        self.params = params
        self._pending: dict = {}

    def backward_input(self, mb, out: torch.Tensor, grad: torch.Tensor | None, inp: torch.Tensor | None):
        self._pending[mb] = (out, grad)
        if inp is None:
            return None
        (dx,) = torch.autograd.grad(out, [inp], grad_outputs=grad, retain_graph=True)
        return dx

    def compute(self, mb) -> None:
        out, grad = self._pending.pop(mb)
        params = [p for p in self.params() if p.requires_grad]
        grads = torch.autograd.grad(out, params, grad_outputs=grad, allow_unused=True)
        with torch.no_grad():
            for p, g in zip(params, grads):
                if g is None:
                    continue
                if p.grad is None:
                    p.grad = g
                else:
                    p.grad.add_(g)

    def pending(self) -> list:
        return sorted(self._pending)

    def clear(self) -> None:
        self._pending.clear()


class KernelWeightGradStore:
    """FIFO of deferred weight-gradient work per model chunk (keys ``(stage, mb)``)."""

    def __init__(self, chunks: dict[int, object]):
        self.chunks = chunks
        self._queue: dict[int, list[tuple[int, Callable[[], None]]]] = {s: [] for s in chunks}

    @contextlib.contextmanager
    def deferring(self, key: tuple[int, int]):
        yield
        self._queue[key[0]].append((key[1], getattr(self.chunks[key[0]], "pop_wgrad", lambda: (lambda: None))()))

    def defer(self, key: tuple[int, int], fn: Callable[[], None]) -> None:
        self._queue[key[0]].append((key[1], fn))

    def compute(self, key: tuple[int, int]) -> None:
        stage, mb = key
        q = self._queue[stage]
        if not q or q[0][0] != mb:
            raise RuntimeError(f"W({mb}) of stage {stage} out of B order {[m for m, _ in q]}: wgrad queues are FIFO")
        _, fn = q.pop(0)
        fn()

    def pending(self) -> list[tuple[int, int]]:
        return [(s, mb) for s, q in self._queue.items() for mb, _ in q]

    def clear(self) -> None:
        for q in self._queue.values():
            q.clear()
