"""Warm handoff: move layer ownership without stopping training (planned / fail-slow
repartition).

1. ``prestage`` at a commit boundary copies parameters and optimizer state of the keys that
   change owner to their destinations.
2. For the next iteration the sources forward the *reduced* gradients of those keys
   (``forward_grads``) and the destinations apply the identical Adam update
   (``lockstep_update``), so destination state stays bit-identical to the source's.
3. Switch to the new plan at the following boundary; no state copy sits on the critical path.
(Reference: ``resihp/state/warm_handoff.py:21-68``.)
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
        self.plan = TransferPlan(transfers=list(plan.transfers))
        self.me, self.comms, self.mgr = me, comms, mgr
        self.specs = specs
        self.old_layout = old_layout
        self.incoming_layout = incoming_layout
        self.kinds = kinds
        self.timeout = timeout
        self.staged: LocalState | None = None

    def _run(self, state: LocalState, kinds, dtype) -> LocalState:
        return execute_transfers(self.plan, self.me, self.comms, self.mgr, specs=self.specs,
                                 old_layout=self.old_layout, old_state=state, new_layout=self.incoming_layout,
                                 kinds=kinds, dtype=dtype, timeout=self.timeout)

    def prestage(self, old_state: LocalState, dtype: torch.dtype) -> LocalState:
        self.staged = self._run(old_state, self.kinds, dtype)
        return self.staged

    def forward_grads(self, reduced_grads: dict[str, torch.Tensor], dtype: torch.dtype) -> dict[str, torch.Tensor]:
        return self._run({"grad": reduced_grads}, ("grad",), dtype)["grad"]

    def lockstep_update(self, grads: dict[str, torch.Tensor], step_count: int, lr: float, betas=(0.9, 0.999),
                        eps: float = 1e-8, weight_decay: float = 0.0) -> None:
        """Apply exactly the update ``runtime.optim.Adam`` applies at ``step_count``."""
        from ..runtime.optim import adam_update_

        assert self.staged is not None, "prestage first"
        for key, g in grads.items():
            adam_update_(self.staged["param"][key], g, self.staged["exp_avg"][key], self.staged["exp_avg_sq"][key],
                         step_count, lr, betas, eps, weight_decay)
