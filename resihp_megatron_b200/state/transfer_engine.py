"""Executes a ``TransferPlan`` for model and optimizer state over the new generation's groups.

Every state kind (parameter, Adam moments, ...) follows the same interval routing, so TP
resharding, PP layer moves and DP replica recovery are one mechanism.  Reused intervals are
copied locally; every remote piece is one isend / irecv per (transfer, kind), tagged
``transfer_index * n_kinds + kind_index``; non-trainable tensors carry only the first kind.  The
old state is only read (it stays valid until the new generation commits).  On GPUs the same
plan is executed by the peer-to-peer migration kernel (``parallel/migration``).
Parity: ``resihp/state/transfer_engine.py:24-59`` (same routing and tag scheme).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .layer_registry import TensorSpec
from .transfer_plan import TransferPlan

LocalState = dict[str, dict[str, torch.Tensor]]
_TAG_SPACE = 2 ** 31 - 1


def _window(t: torch.Tensor, spec: TensorSpec, held: tuple[int, int], span: tuple[int, int]) -> torch.Tensor:
    """The part of ``t`` (which holds interval ``held``) that covers ``span``."""
    if spec.dim is None:
        return t
    return t.narrow(spec.dim, span[0] - held[0], span[1] - span[0])


def execute_transfers(plan: TransferPlan, me: str, comms, mgr, *, specs: dict[str, TensorSpec],
                      old_layout: dict[str, tuple[int, int]], old_state: LocalState,
                      new_layout: dict[str, tuple[int, int]], kinds: tuple[str, ...], dtype: torch.dtype,
                      device: str = "cpu", timeout: float = 300.0) -> LocalState:
    def carried(key: str) -> tuple[str, ...]:
        return kinds if specs[key].trainable else kinds[:1]

    fresh: LocalState = {kind: {} for kind in kinds}
    for key, span in new_layout.items():
        for kind in carried(key):
            fresh[kind][key] = torch.empty(specs[key].local_shape(span), dtype=dtype, device=device)
    for dst, key, span in (r for r in plan.reuse if r[0] == me):
        for kind in carried(key):
            _window(fresh[kind][key], specs[key], new_layout[key], span).copy_(
                _window(old_state[kind][key], specs[key], old_layout[key], span))
    pending, arrivals = [], []
    for i, t in enumerate(plan.transfers):
        if me not in (t.src, t.dst):
            continue
        spec = specs[t.key]
        for j, kind in enumerate(carried(t.key)):
            tag = (i * len(kinds) + j) % _TAG_SPACE
            if t.src == me:
                outgoing = _window(old_state[kind][t.key], spec, old_layout[t.key], t.interval).contiguous()
                pending.append((dist.isend(outgoing, comms.rank_of(t.dst), tag=tag), outgoing))
            if t.dst == me:
                incoming = torch.empty(spec.local_shape(t.interval), dtype=dtype, device=device)
                pending.append((dist.irecv(incoming, comms.rank_of(t.src), tag=tag), incoming))
                arrivals.append((incoming, kind, t.key, t.interval))
    for work, _buffer in pending:
        mgr.guarded_wait(work, timeout=timeout, what="state transfer")
    for incoming, kind, key, span in arrivals:
        _window(fresh[kind][key], specs[key], new_layout[key], span).copy_(incoming)
    return fresh
