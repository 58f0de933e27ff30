"""Peer-to-peer execution of a state transfer plan on one NVLink/NVSwitch node.

Every rank of the new generation stages the state it held under the old plan (per key and kind,
fp32, packed in an order every rank derives from the old holdings alone) into a symmetric peer
heap.  After a bounded barrier each rank issues one strided-copy launch (``symm_copy2d``) that
pulls every slice it holds under the new plan -- from its own staging area or a peer's, over
NVLink -- straight into its new tensors; a column block of a row-parallel weight is a strided
copy, not a gather into a contiguous buffer.  A second barrier releases the staging heaps.  This
replaces the transfer engine's one NCCL send/receive per (slice, kind)
(``state/transfer_engine.py``; reference: ``resihp/state/transfer_engine.py:24-59``).
"""

from __future__ import annotations

import math

import torch

from ..ops._build import ext
from ..state.layer_registry import Holdings, TensorSpec, device_layout
from ..state.transfer_plan import TransferPlan
from .symm import AbortWord, SymmetricHeap

ALIGN = 256


def pack_table(h: Holdings, device: str, specs: dict[str, TensorSpec],
               kinds: tuple[str, ...]) -> tuple[dict[tuple[str, str], int], int]:
    """Byte offset of every (key, kind) ``device`` holds under ``h`` in its staging area, and the
    area's size.  Keys in sorted order, kinds in ``kinds`` order (non-trainable keys: first kind)."""
    table: dict[tuple[str, str], int] = {}
    off = 0
    for key, iv in sorted(device_layout(h, device).items()):
        spec = specs[key]
        n = math.prod(spec.local_shape(iv))
        for kind in (kinds if spec.trainable else kinds[:1]):
            table[(key, kind)] = off
            off += (n * 4 + ALIGN - 1) // ALIGN * ALIGN
    return table, off


def _geometry(spec: TensorSpec, iv: tuple[int, int], held: tuple[int, int]) -> tuple[int, int, int, int]:
    """``(rows, row_bytes, pitch_bytes, offset_bytes)`` of interval ``iv`` inside a local tensor
    that holds ``held`` of the key (fp32, row-major)."""
    shape = spec.local_shape(held)
    if spec.dim is None:
        n = math.prod(shape) * 4
        return 1, n, n, 0
    inner = math.prod(shape[spec.dim + 1:])
    outer = math.prod(shape[:spec.dim])
    return outer, (iv[1] - iv[0]) * inner * 4, shape[spec.dim] * inner * 4, (iv[0] - held[0]) * inner * 4


def migrate_p2p(plan: TransferPlan, me: str, world: list[str], *, specs: dict[str, TensorSpec], old_h: Holdings,
                new_h: Holdings, old_state: dict[str, dict[str, torch.Tensor]],
                new_state: dict[str, dict[str, torch.Tensor]], kinds: tuple[str, ...], device, exchange=None,
                abort: AbortWord | None = None, budget_s: float = 60.0, _heap: SymmetricHeap | None = None,
                _stage: bool = True, _copy: bool = True) -> int:
    """Fill ``new_state[kind][key]`` (contiguous fp32 tensors of this rank's new local shapes)
    from the old holders' staged state.  Collective over ``world`` (the new generation's
    devices, ``exchange`` all-gathers the heap handles in that order).  Returns the bytes this
    rank pulled.  ``_heap`` / ``_stage`` / ``_copy``: emulated ranks in one process (tests)."""
    dev = torch.device(device)
    rank = world.index(me)
    tables = {d: pack_table(old_h, d, specs, kinds) for d in world}
    cap = max(t[1] for t in tables.values())
    heap = _heap or SymmetricHeap({"stage": (max(cap, ALIGN) // 4, torch.float32)}, rank, len(world), exchange, dev,
                                  abort)
    emulated = _heap is not None
    base = heap.peer_ptrs("stage")
    if _stage:
        stage = heap.tensor("stage")
        for (key, kind), off in tables[me][0].items():
            t = old_state.get(kind, {}).get(key)
            if t is None:  # held under the old plan but not up to date: never chosen as a source
                continue
            stage[off // 4: off // 4 + t.numel()].copy_(t.reshape(-1))
        if not emulated:
            heap.barrier(budget_s)
    pulled = 0
    if _copy:
        new_layout = device_layout(new_h, me)
        six: list[int] = []
        moves = [(tr.src, tr.key, tr.interval) for tr in plan.transfers if tr.dst == me]
        moves += [(me, key, iv) for dst, key, iv in plan.reuse if dst == me]
        for src, key, iv in moves:
            spec = specs[key]
            held_src = device_layout(old_h, src)[key]
            rows, row_bytes, sp, so = _geometry(spec, iv, held_src)
            _, _, dp, do = _geometry(spec, iv, new_layout[key])
            for kind in (kinds if spec.trainable else kinds[:1]):
                dst = new_state[kind][key]
                if not dst.is_contiguous():
                    raise ValueError(f"{key}/{kind}: the destination must be contiguous")
                six += [base[world.index(src)] + tables[src][0][(key, kind)] + so, dst.data_ptr() + do, rows,
                        row_bytes, sp, dp]
                pulled += rows * row_bytes
        if six:
            ext().symm_copy2d(six, dev.index if dev.index is not None else 0)
        if not emulated:
            heap.barrier(budget_s)  # nobody reads this rank's staging area any more
            heap.check()
            heap.close()
    return pulled
