"""Price of a plan transition -- the ``buy`` side of the ski-rental policy.

Replays the slice-level transfer plan the workers would execute between two plans (local
reuse, striping, locality), charges each device the time of the bytes it sends or receives,
and adds the communicator rebuild time.  ``bytes_per_elem`` defaults to 14 (bf16 weight +
fp32 master + two fp32 Adam moments).  (Reference: ``resihp/plan/reconfig_cost.py:28-73``.)
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass

from .hetero_plan import HeteroParallelPlan
from .model_spec import ModelSpec
from ..state.layer_registry import TensorSpec, holdings
from ..state.transfer_plan import plan_transfers


@dataclass(frozen=True)
class ReconfigEstimate:
    seconds: float
    bytes_moved: int
    max_device_bytes: int
    rebuild_s: float


def gpt_layer_specs(model: ModelSpec) -> dict[str, TensorSpec]:
    """Per-layer tensors of a GPT layer with their TP partition dimension."""
    h, f = model.hidden, model.ffn
    hd = h // model.num_heads
    qkv = h + 2 * model.num_kv_heads * hd
    fc1 = (2 if model.swiglu else 1) * f
    specs = {}
    for l in range(model.num_layers):
        for name, shape, dim in (("attn.qkv.weight", (qkv, h), 0), ("attn.proj.weight", (h, h), 1),
                                 ("mlp.fc1.weight", (fc1, h), 0), ("mlp.fc2.weight", (h, f), 1),
                                 ("ln1.weight", (h,), None), ("ln2.weight", (h,), None)):
            key = f"layers.{l}.{name}"
            specs[key] = TensorSpec(key, shape, dim)
    return specs


def layer_of_key(key: str) -> int:
    return int(key.split(".")[1])


def estimate_reconfig_cost(old: HeteroParallelPlan | None, new: HeteroParallelPlan, specs: dict[str, TensorSpec], *,
                           bytes_per_elem: int = 14, inter_bw: float = 25e9, intra_bw: float = 300e9,
                           rebuild_s: float = 2.0, node_of: dict[str, str] | None = None) -> ReconfigEstimate:
    if old is None:
        return ReconfigEstimate(rebuild_s, 0, 0, rebuild_s)
    node_of = node_of or {}
    plan = plan_transfers(holdings(old, specs, layer_of_key), holdings(new, specs, layer_of_key),
                          valid_sources=set(old.world) & set(new.world), node_of=node_of)
    busy_s: dict[str, float] = defaultdict(float)
    busy_b: dict[str, int] = defaultdict(int)
    total = 0
    for t in plan.transfers:
        n = 1
        for d in specs[t.key].local_shape(t.interval):
            n *= d
        b = n * bytes_per_elem
        local = node_of.get(t.src) is not None and node_of.get(t.src) == node_of.get(t.dst)
        secs = b / (intra_bw if local else inter_bw)
        for dev in (t.src, t.dst):
            busy_s[dev] += secs
            busy_b[dev] += b
        total += b
    return ReconfigEstimate(rebuild_s + max(busy_s.values(), default=0.0), total, max(busy_b.values(), default=0),
                            rebuild_s)
