"""Logical tensors of the GPU Llama model, and export / import of one rank's training state.

Every tensor of ``models.tp_stage`` has a layout-independent key (``embed``,
``layers.<l>.<attn_norm|mlp_norm|wq|wk|wv|wo|w1|w3|w2>``, ``final_norm``, ``lm_head``) with its
global shape and tensor-parallel dimension, so ``state.layer_registry.holdings`` derives who
holds which interval of every key under any plan, and ``state.transfer_plan`` the slices a
reconfiguration moves -- the same machinery as the CPU runtime's.

``export_state`` gives a rank's per-key fp32 master weights and Adam moments (ZeRO-1 shards are
first all-gathered inside each data-parallel group, as the reference does for Megatron's
distributed optimizer: ``resihp/state/megatron_adapter.py:21-53``); ``import_state`` writes a
migrated state into a new runtime's flat buffers (optimizer shard slices, and the bf16 compute
copy of every weight).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.config import GPTConfig
from ..state.layer_registry import FULL, TensorSpec

KINDS = ("param", "exp_avg", "exp_avg_sq")


def gpu_tensor_specs(cfg: GPTConfig, fp8_history: int = 0) -> dict[str, TensorSpec]:
    """Every logical tensor; ``fp8_history`` > 0 adds each layer's fp8 amax history
    (``layers.<l>.amax_history``, ``[12, fp8_history]``, replicated, no optimizer state)."""
    from ..models.fp8_linear import NSLOTS

    H, D, F, V = cfg.hidden, cfg.head_dim, cfg.ffn, cfg.vocab_size
    q, kv = cfg.heads * D, cfg.kv_heads * D
    out = {"embed": TensorSpec("embed", (V, H), None)}
    mlp = (("w1", (F, H), 0),) + ((("w3", (F, H), 0),) if cfg.gated else ()) + (("w2", (H, F), 1),)
    for l in range(cfg.layers):
        p = f"layers.{l}."
        for name, shape, dim in (("attn_norm", (H,), None), ("mlp_norm", (H,), None), ("wq", (q, H), 0),
                                 ("wk", (kv, H), 0), ("wv", (kv, H), 0), ("wo", (H, q), 1)) + mlp:
            out[p + name] = TensorSpec(p + name, shape, dim)
        if fp8_history:
            out[p + "amax_history"] = TensorSpec(p + "amax_history", (NSLOTS, fp8_history), None, trainable=False)
    out["final_norm"] = TensorSpec("final_norm", (H,), None)
    out["lm_head"] = TensorSpec("lm_head", (V, H), None)
    return out


def gpu_layer_of(num_layers: int):
    """Layer a key belongs to (the embedding to the first, the head to the last)."""

    def layer_of(key: str) -> int:
        if key == "embed":
            return 0
        if key in ("final_norm", "lm_head"):
            return num_layers - 1
        return int(key.split(".")[1])

    return layer_of


def partition_sizes(cfg: GPTConfig) -> tuple[int, ...]:
    """Lengths of the tensor-parallel dimensions (query heads, key/value heads, FFN)."""
    return tuple(sorted({cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn}))


def _sets(rt):
    return rt.param_sets()


def _buffers(rt) -> dict[str, torch.Tensor]:
    """Non-trainable per-layer state of the runtime (fp8 amax histories), by logical key."""
    return rt.buffers() if hasattr(rt, "buffers") else {}


def export_state(rt) -> tuple[dict[str, dict[str, torch.Tensor]], dict[str, tuple[int, int]]]:
    """``(state, layout)``: ``state[kind][key]`` fp32 tensors of this rank's local shape and
    ``layout[key]`` its interval along the key's TP dimension.  Collective over every
    data-parallel group whose optimizer state is sharded."""
    state: dict[str, dict[str, torch.Tensor]] = {k: {} for k in KINDS}
    layout: dict[str, tuple[int, int]] = {}
    for P, sync in _sets(rt):
        bufs = (P.master, P.exp_avg, P.exp_avg_sq)
        if P.shard_count > 1:
            full = []
            for b in bufs:
                t = torch.empty(P.numel, dtype=torch.float32, device=b.device)
                sync.wait(dist.all_gather_into_tensor(t, b, group=sync.group, async_op=True))
                full.append(t)
            bufs = tuple(full)
        for name in P.order:
            s, o = P.specs[name], P.offsets[name]
            for kind, b in zip(KINDS, bufs):
                state[kind][name] = b[o:o + s.numel].view(s.shape)
            layout[name] = s.shard_range if s.shard_dim is not None else FULL
    for key, t in _buffers(rt).items():
        state["param"][key] = t.clone()
        layout[key] = FULL
    return state, layout


def import_state(rt, state: dict[str, dict[str, torch.Tensor]], step: int) -> None:
    """Load migrated per-key state into ``rt``'s flat buffers (this rank's optimizer shard and
    the full bf16 compute weights) and set the optimizer step count."""
    for P, _ in _sets(rt):
        for name in P.order:
            w = state["param"][name]
            P.w(name).copy_(w)
            piece = P.owned_piece(name)
            if piece is None:
                continue
            a, b, n = piece
            for kind, buf in zip(KINDS, (P.master, P.exp_avg, P.exp_avg_sq)):
                buf[b:b + n].copy_(state[kind][name].reshape(-1)[a:a + n])
        P.step = step
    for key, t in _buffers(rt).items():
        if key in state["param"]:
            t.copy_(state["param"][key])


def local_layout(rt) -> dict[str, tuple[int, int]]:
    """Interval of every key this rank holds (its TP dimension; ``FULL`` when replicated)."""
    out = {}
    for P, _ in _sets(rt):
        for name in P.order:
            s = P.specs[name]
            out[name] = tuple(s.shard_range) if s.shard_dim is not None else FULL
    for key in _buffers(rt):
        out[key] = FULL
    return out


def checkpoint_slices(rt, specs: dict[str, TensorSpec]):
    """This rank's state as checkpoint slices ``[(SliceMeta, {kind: tensor})]`` (collective over
    ZeRO-sharded data-parallel groups, like ``export_state``)."""
    from ..state.checkpoint import SliceMeta

    state, layout = export_state(rt)
    return [(SliceMeta(key, specs[key].global_shape, specs[key].dim, tuple(iv)),
             {k: state[k][key] for k in (KINDS if specs[key].trainable else KINDS[:1])})
            for key, iv in layout.items()]


def load_checkpoint_into(rt, checkpointer, iteration: int, specs: dict[str, TensorSpec]) -> None:
    """Assemble this rank's slices of every key from checkpoint ``iteration`` (whatever layout
    wrote it: reshard on load) and load them; the optimizer step count becomes ``iteration + 1``."""
    from ..state.checkpoint import SliceMeta

    wanted = [SliceMeta(key, specs[key].global_shape, specs[key].dim, iv) for key, iv in local_layout(rt).items()]
    got = checkpointer.load(iteration, [w for w in wanted if specs[w.key].trainable], KINDS)
    got.update(checkpointer.load(iteration, [w for w in wanted if not specs[w.key].trainable], KINDS[:1]))
    dev = rt.device
    state = {k: {key: got[key][k].to(dev) for key in got if k in got[key]} for k in KINDS}
    import_state(rt, state, step=iteration + 1)
