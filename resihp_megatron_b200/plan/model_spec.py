"""Model shape, memory model and compute-cost profile used by the planner and the detector.

``ModelSpec`` gives parameter counts, TP feasibility and the per-GPU memory model (weights +
fp32 grads + optimizer state / dp_shard, plus stored activations per in-flight micro-batch:
34 * s * b * h bytes per layer, divided by TP under sequence parallelism).  ``ModelProfile`` is
the per-layer cost at TP=1 on a healthy device, ``T_fwd = alpha * N + beta * sum(l_i^2)`` --
the same model the online RLS predictor fits, so prediction and planning agree.  On B200 the
profile is fitted from device timings of this package's kernels (``from_gpu_measurement``).
(Reference: ``resihp/plan/model_spec.py:9-83``.)
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ModelSpec:
    num_layers: int
    hidden: int
    ffn: int
    num_heads: int
    num_kv_heads: int
    vocab: int
    seq_len: int
    micro_batch_size: int = 1
    param_bytes: int = 2
    grad_bytes: int = 4
    optim_bytes: int = 12
    swiglu: bool = True

    def layer_params(self) -> int:
        hd = self.hidden // self.num_heads
        attn = 2 * self.hidden * self.hidden + 2 * self.hidden * self.num_kv_heads * hd
        mlp = (3 if self.swiglu else 2) * self.hidden * self.ffn
        return attn + mlp + 2 * self.hidden

    def embedding_params(self) -> int:
        return self.vocab * self.hidden

    def tp_feasible(self, k: int) -> bool:
        return k >= 1 and self.num_heads % k == 0 and self.num_kv_heads % k == 0 and self.ffn % k == 0

    def static_bytes(self, layers: int, tp: int, dp_shard: int = 1, extra_params: int = 0) -> float:
        p = (layers * self.layer_params() + extra_params) / tp
        return p * (self.param_bytes + self.grad_bytes) + p * self.optim_bytes / dp_shard

    def activation_bytes(self, layers: int, tp: int, sequence_parallel: bool = True) -> float:
        sbh = self.seq_len * self.micro_batch_size * self.hidden
        return layers * sbh * 34 / (tp if sequence_parallel else 1)

    def boundary_bytes(self) -> int:
        """bf16 hidden state crossing a pipeline boundary."""
        return self.seq_len * self.micro_batch_size * self.hidden * 2

    @staticmethod
    def from_config(cfg, micro_batch_size: int = 1) -> "ModelSpec":
        """From a ``models.config.GPTConfig``."""
        return ModelSpec(cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.vocab_size, cfg.seq_len,
                         micro_batch_size)


@dataclass(frozen=True)
class ModelProfile:
    alpha: float
    beta: float
    bwd_ratio: float = 2.0
    w_fraction: float = 0.5
    tp_overhead: float = 0.04
    p2p_bandwidth: float = 25e9
    p2p_latency: float = 20e-6
    intra_node_bandwidth: float = 300e9
    first_stage_extra_layers: float = 0.0
    last_stage_extra_layers: float = 1.0
    grad_sync_overlap: float = 0.8

    def tp_efficiency(self, k: int) -> float:
        return 1.0 / (1.0 + self.tp_overhead * (k - 1))

    def fwd_layer_time(self, tokens: float, sum_sq: float, tp: int, speed: float) -> float:
        return (self.alpha * tokens + self.beta * sum_sq) / (tp * self.tp_efficiency(tp) * max(speed, 1e-9))

    def group_speed(self, tp: int, min_speed: float) -> float:
        """Relative throughput of a TP group: ``k * min p`` times the TP scaling efficiency."""
        return tp * self.tp_efficiency(tp) * min_speed

    def p2p_time(self, nbytes: float, same_node: bool = False) -> float:
        return self.p2p_latency + nbytes / (self.intra_node_bandwidth if same_node else self.p2p_bandwidth)

    @staticmethod
    def b200(spec: ModelSpec, sustained_tflops: float = 1000.0, attn_tflops: float = 400.0) -> "ModelProfile":
        """Analytic B200 profile: per-layer forward time from dense matmul FLOPs at the sustained
        GEMM rate (alpha, per token) and causal attention FLOPs at the attention rate (beta,
        per squared token); NVLink 5 (~770 GB/s measured per direction) for every peer of a
        node, 400 Gb/s-class NICs between nodes."""
        hd = spec.hidden // spec.num_heads
        mm = 2 * (spec.layer_params() - 2 * spec.hidden)
        alpha = mm / (sustained_tflops * 1e12)
        beta = (2 * spec.num_heads * hd) / (attn_tflops * 1e12)  # QK^T + PV, causal half of 4*h*d
        return ModelProfile(alpha=alpha, beta=beta, p2p_bandwidth=50e9, intra_node_bandwidth=770e9,
                            p2p_latency=10e-6)
