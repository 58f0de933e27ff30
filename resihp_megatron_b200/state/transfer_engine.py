"""Executes a ``TransferPlan`` for model and optimizer state over the new generation's groups.

Every kind (parameter, Adam moments, ...) follows the same interval routing, so TP
resharding, PP layer moves and DP replica recovery are one mechanism.  Reused intervals are
copied locally; every remote piece is one isend/irecv per (transfer, kind) with tag
``i * n_kinds + j``; non-trainable tensors carry only the first kind.  The old state is never
modified (it stays valid until the new generation commits).  On GPU the same plan is executed by
the peer-to-peer migration kernel (``parallel/migration``).
(Reference: ``resihp/state/transfer_engine.py:24-59``.)
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .layer_registry import TensorSpec
from .transfer_plan import TransferPlan

LocalState = dict[str, dict[str, torch.Tensor]]


def _view(t: torch.Tensor, spec: TensorSpec, have: tuple[int, int], want: tuple[int, int]) -> torch.Tensor:
    if spec.dim is None:
        return t
    return t.narrow(spec.dim, want[0] - have[0], want[1] - want[0])


def execute_transfers(plan: TransferPlan, me: str, comms, mgr, *, specs: dict[str, TensorSpec],
                      old_layout: dict[str, tuple[int, int]], old_state: LocalState,
                      new_layout: dict[str, tuple[int, int]], kinds: tuple[str, ...], dtype: torch.dtype,
                      device: str = "cpu", timeout: float = 300.0) -> LocalState:
    def kinds_of(key: str) -> tuple[str, ...]:
        return kinds if specs[key].trainable else kinds[:1]

    new: LocalState = {k: {} for k in kinds}
    for key, iv in new_layout.items():
        for k in kinds_of(key):
            new[k][key] = torch.empty(specs[key].local_shape(iv), dtype=dtype, device=device)
    for dst, key, iv in plan.reuse:
        if dst == me:
            for k in kinds_of(key):
                _view(new[k][key], specs[key], new_layout[key], iv).copy_(
                    _view(old_state[k][key], specs[key], old_layout[key], iv))
    nk = len(kinds)
    works: list = []
    landed: list[tuple[torch.Tensor, str, str, tuple[int, int]]] = []
    for i, tr in enumerate(plan.transfers):
        spec = specs[tr.key]
        for j, k in enumerate(kinds_of(tr.key)):
            tag = (i * nk + j) % (2 ** 31 - 1)
            if tr.src == me:
                piece = _view(old_state[k][tr.key], spec, old_layout[tr.key], tr.interval).contiguous()
                works.append((dist.isend(piece, comms.rank_of(tr.dst), tag=tag), piece))
            if tr.dst == me:
                buf = torch.empty(spec.local_shape(tr.interval), dtype=dtype, device=device)
                works.append((dist.irecv(buf, comms.rank_of(tr.src), tag=tag), buf))
                landed.append((buf, k, tr.key, tr.interval))
    for work, _ in works:
        mgr.guarded_wait(work, timeout=timeout, what="state transfer")
    for buf, k, key, iv in landed:
        _view(new[k][key], specs[key], new_layout[key], iv).copy_(buf)
    return new
