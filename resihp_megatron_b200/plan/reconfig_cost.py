"""What a plan transition costs -- the ``buy`` price of the ski-rental policy.

The estimate replays the slice-level transfer plan the workers would execute between the two
plans (with local reuse, striping across holders and locality), charges every device for the
bytes it sends or receives at the intra- or inter-node bandwidth, takes the busiest device as
the migration time and adds the communicator rebuild.  ``bytes_per_elem`` defaults to 14: a
bf16 weight, its fp32 master copy and two fp32 Adam moments.
Parity: ``resihp/plan/reconfig_cost.py:28-73`` (same pricing model).
"""

from __future__ import annotations

import math
from collections import Counter
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


# (registry name, rows, cols, TP partition dim) of one decoder layer; None cols = a vector
def _layer_tensors(model: ModelSpec):
    h = model.hidden
    kv = model.num_kv_heads * (h // model.num_heads)
    up = model.ffn * (2 if model.swiglu else 1)
    yield "attn.qkv.weight", (h + 2 * kv, h), 0
    yield "attn.proj.weight", (h, h), 1
    yield "mlp.fc1.weight", (up, h), 0
    yield "mlp.fc2.weight", (h, model.ffn), 1
    yield "ln1.weight", (h,), None
    yield "ln2.weight", (h,), None


def gpt_layer_specs(model: ModelSpec) -> dict[str, TensorSpec]:
    """Registry specs of every layer's tensors, keyed ``layers.{l}.{name}``."""
    out = {}
    for layer in range(model.num_layers):
        for name, shape, dim in _layer_tensors(model):
            key = f"layers.{layer}.{name}"
            out[key] = TensorSpec(key, shape, dim)
    return out


def layer_of_key(key: str) -> int:
    return int(key.split(".")[1])


def estimate_reconfig_cost(old: HeteroParallelPlan | None, new: HeteroParallelPlan, specs: dict[str, TensorSpec], *,
                           bytes_per_elem: int = 14, inter_bw: float = 25e9, intra_bw: float = 300e9,
                           rebuild_s: float = 2.0, node_of: dict[str, str] | None = None) -> ReconfigEstimate:
    if old is None:  # a fresh start moves no state
        return ReconfigEstimate(rebuild_s, 0, 0, rebuild_s)
    where = node_of or {}
    transfers = plan_transfers(holdings(old, specs, layer_of_key), holdings(new, specs, layer_of_key),
                               valid_sources=set(old.world) & set(new.world), node_of=where).transfers
    seconds_of, bytes_of = Counter(), Counter()
    for t in transfers:
        nbytes = bytes_per_elem * math.prod(specs[t.key].local_shape(t.interval))
        same_node = where.get(t.src) is not None and where.get(t.src) == where.get(t.dst)
        secs = nbytes / (intra_bw if same_node else inter_bw)
        for dev in (t.src, t.dst):  # a copy occupies both ends
            seconds_of[dev] += secs
            bytes_of[dev] += nbytes
    busiest = max(seconds_of.values(), default=0.0)
    return ReconfigEstimate(rebuild_s + busiest, sum(bytes_of.values()) // 2, max(bytes_of.values(), default=0),
                            rebuild_s)
