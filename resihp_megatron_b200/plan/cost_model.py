"""Binds a plan to the model profile, the workload and the device speeds, and prices each
schedulable operation for the pipeline simulator.

* Compute: the forward of micro-batch ``m`` on group ``(r, s)`` costs
  ``weight_s * (alpha * tokens_m + beta * sum_sq_m) / speed_(r,s)`` where ``weight_s`` is the
  stage's layer count plus the embedding / head work charged to the first and last stage, and
  ``speed`` is the group's throughput (slowest member x TP efficiency x CP degree).  Backward is
  ``bwd_ratio`` times the forward; with a split backward (zero bubble), B keeps
  ``1 - w_fraction`` of it and W the rest.
* Pipeline messages: latency + bytes / bandwidth (intra- or inter-node), plus an intra-TP
  all-gather when the two sides' TP degrees differ without sequence parallelism.
* DP gradient sync: the non-overlapped part of a ring all-reduce of the stage's shard.
Parity: ``resihp/plan/cost_model.py:14-81`` (same cost terms).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .hetero_plan import HeteroParallelPlan
from .model_spec import ModelProfile, ModelSpec

Key = tuple[int, int]


@dataclass(frozen=True)
class Workload:
    """Per micro-batch token count ``N`` and attention work ``sum(l_i^2)`` (packed documents)."""

    tokens: tuple[float, ...]
    sum_sq: tuple[float, ...]

    @classmethod
    def uniform(cls, num_microbatches: int, seq_len: int, micro_batch_size: int = 1) -> "Workload":
        per_mb_tokens = float(seq_len * micro_batch_size)
        per_mb_sq = float(micro_batch_size) * float(seq_len) * float(seq_len)
        return cls(tuple([per_mb_tokens] * num_microbatches), tuple([per_mb_sq] * num_microbatches))

    @classmethod
    def from_doc_lengths(cls, docs: list[list[int]]) -> "Workload":
        tokens = tuple(float(sum(mb)) for mb in docs)
        squares = tuple(float(sum(n * n for n in mb)) for mb in docs)
        return cls(tokens, squares)

    def work(self, profile: ModelProfile, mb: int) -> float:
        return profile.alpha * self.tokens[mb] + profile.beta * self.sum_sq[mb]


@dataclass
class CostModel:
    plan: HeteroParallelPlan
    model: ModelSpec
    profile: ModelProfile
    workload: Workload
    speeds: dict[str, float]
    node_of: dict[str, str]
    split_backward: bool = False
    _stage_weight: list = field(init=False, repr=False)
    _speed_cache: dict = field(init=False, repr=False, default_factory=dict)

    def __post_init__(self) -> None:
        last = self.plan.num_stages - 1
        self._stage_weight = []
        for s, (lo, hi) in enumerate(self.plan.layer_partition()):
            extra = (self.profile.first_stage_extra_layers if s == 0 else 0.0) + \
                    (self.profile.last_stage_extra_layers if s == last else 0.0)
            self._stage_weight.append((hi - lo) + extra)

    def group_speed(self, key: Key) -> float:
        if key not in self._speed_cache:
            g = self.plan.group(*key)
            slowest = min(self.speeds.get(d, 1.0) for d in g.devices)
            self._speed_cache[key] = g.cp * self.profile.group_speed(g.tp, slowest)
        return self._speed_cache[key]

    def fwd(self, key: Key, mb: int) -> float:
        return self._stage_weight[key[1]] * self.workload.work(self.profile, mb) / max(self.group_speed(key), 1e-12)

    def cost(self, key: Key, op: str, mb: int) -> float:
        """Seconds for op ``F``, ``B`` or ``W`` of micro-batch ``mb`` on group ``key``."""
        forward = self.fwd(key, mb)
        if op == "F":
            return forward
        backward = forward * self.profile.bwd_ratio
        w_part = backward * self.profile.w_fraction
        if op == "W":
            return w_part
        return backward - w_part if self.split_backward else backward

    def _nodes(self, key: Key) -> set:
        return {self.node_of.get(d) for d in self.plan.group(*key).devices}

    def comm(self, src: Key, dst: Key, kind: str) -> float:
        """Seconds to move one boundary activation (or its gradient) from ``src`` to ``dst``."""
        nbytes = self.model.boundary_bytes()
        seconds = self.profile.p2p_time(nbytes, same_node=self._nodes(src) == self._nodes(dst))
        reshaped = self.plan.group(*src).tp != self.plan.group(*dst).tp
        if reshaped and not self.plan.sequence_parallel:
            seconds += nbytes / self.profile.intra_node_bandwidth  # receivers re-gather inside TP
        return seconds

    def sync_time(self, key: Key) -> float:
        """Non-overlapped seconds of the stage's DP gradient all-reduce (ring) for group ``key``."""
        replicas = len(self.plan.groups_at(key[1]))
        if replicas <= 1:
            return 0.0
        lo, hi = self.plan.layer_partition()[key[1]]
        shard_bytes = (hi - lo) * self.model.layer_params() * self.model.grad_bytes / self.plan.group(*key).tp
        ring_seconds = 2.0 * (replicas - 1) / replicas * shard_bytes / self.profile.p2p_bandwidth
        return (1.0 - self.profile.grad_sync_overlap) * ring_seconds
