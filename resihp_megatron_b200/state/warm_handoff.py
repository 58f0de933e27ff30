"""Warm handoff: move layer ownership without stopping training (planned or fail-slow
repartition).

1. At a commit boundary ``prestage`` copies the parameters and optimizer state of the keys that
   change owner to their new owners.
2. During the next iteration the old owners forward the *reduced* gradients of those keys
   (``forward_grads``) and the new owners apply the identical Adam update (``lockstep_update``),
   so their copies stay bit-identical to the old owners'.
3. The plan switches at the following boundary; no state copy sits on the critical path.
Parity: ``resihp/state/warm_handoff.py:21-68`` (same three steps).
"""

from __future__ import annotations

import torch

from .layer_registry import TensorSpec
from .transfer_engine import LocalState, execute_transfers
from .transfer_plan import TransferPlan


class WarmHandoff:
    def __init__(self, plan: TransferPlan, me: str, comms, mgr, specs: dict[str, TensorSpec],
                 old_layout: dict[str, tuple[int, int]], incoming_layout: dict[str, tuple[int, int]],
                 kinds: tuple[str, ...] = ("param", "exp_avg", "exp_avg_sq"), timeout: float = 300.0):
        self.plan = TransferPlan(transfers=list(plan.transfers))  # moves only: nothing is reused in place
        self.me, self.comms, self.mgr, self.specs = me, comms, mgr, specs
        self.old_layout, self.incoming_layout = old_layout, incoming_layout
        self.kinds, self.timeout = kinds, timeout
        self.staged: LocalState | None = None

    def _move(self, state: LocalState, kinds: tuple[str, ...], dtype: torch.dtype) -> LocalState:
        return execute_transfers(self.plan, self.me, self.comms, self.mgr, specs=self.specs, old_layout=self.old_layout,
                                 old_state=state, new_layout=self.incoming_layout, kinds=kinds, dtype=dtype,
                                 timeout=self.timeout)

    def prestage(self, old_state: LocalState, dtype: torch.dtype) -> LocalState:
        self.staged = self._move(old_state, self.kinds, dtype)
        return self.staged

    def forward_grads(self, reduced_grads: dict[str, torch.Tensor], dtype: torch.dtype) -> dict[str, torch.Tensor]:
        return self._move({"grad": reduced_grads}, ("grad",), dtype)["grad"]

    def lockstep_update(self, grads: dict[str, torch.Tensor], step_count: int, lr: float, betas=(0.9, 0.999),
                        eps: float = 1e-8, weight_decay: float = 0.0) -> None:
        """Apply exactly the update ``runtime.optim.Adam`` applies at ``step_count``."""
        from ..runtime.optim import adam_update_

        if self.staged is None:
            raise RuntimeError("prestage first")
        staged = self.staged
        for key, grad in grads.items():
            adam_update_(staged["param"][key], grad, staged["exp_avg"][key], staged["exp_avg_sq"][key], step_count,
                         lr, betas, eps, weight_decay)
