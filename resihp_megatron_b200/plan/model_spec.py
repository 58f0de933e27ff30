"""Model shape, per-GPU memory model and compute-cost profile, shared by the planner and the
fail-slow detector.

``ModelSpec`` answers three questions about a decoder: how many parameters a layer has, which
TP degrees divide it, and how many bytes a pipeline stage needs per GPU (weights and fp32
gradients, optimizer state divided over a ZeRO-1 group, and the stored activations of every
micro-batch in flight -- 34 bytes per token per hidden unit and layer, the flash-attention
figure of Korthikanti et al., "Reducing Activation Recomputation in Large Transformer Models",
divided by TP under sequence parallelism).

``ModelProfile`` is the per-layer forward cost on one healthy GPU at TP=1,
``t = alpha * tokens + beta * sum(doc_len^2)`` (dense GEMMs scale with tokens, causal attention
with the squared document lengths), the TP scaling overhead and the link model.  The online RLS
predictor fits the same two-term model, so planning and detection agree.  ``b200`` derives it
analytically from kernel rates; ``fit`` derives it from measured forward times of this
package's kernels (least squares), which anchors the planner's predictions to the hardware.
Parity: ``resihp/plan/model_spec.py:9-83`` (same fields and formulas).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

# bytes of stored activations per (token x hidden unit) of one layer, flash attention, bf16
ACTIVATION_BYTES_PER_TOKEN_HIDDEN = 34


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

    @property
    def head_dim(self) -> int:
        return self.hidden // self.num_heads

    @property
    def tokens_per_microbatch(self) -> int:
        return self.seq_len * self.micro_batch_size

    def layer_params(self) -> int:
        h, kv = self.hidden, self.num_kv_heads * self.head_dim
        attention = h * (2 * h + 2 * kv)  # wq, wo: h x h; wk, wv: h x kv
        mlp = h * self.ffn * (3 if self.swiglu else 2)
        norms = 2 * h
        return attention + mlp + norms

    def embedding_params(self) -> int:
        return self.vocab * self.hidden

    def tp_feasible(self, k: int) -> bool:
        """Megatron's TP layout needs ``k`` to divide the query heads, the KV heads and the FFN."""
        return k >= 1 and all(n % k == 0 for n in (self.num_heads, self.num_kv_heads, self.ffn))

    def _bytes_per_param(self, dp_shard: int) -> float:
        return self.param_bytes + self.grad_bytes + self.optim_bytes / dp_shard

    def static_bytes(self, layers: int, tp: int, dp_shard: int = 1, extra_params: int = 0) -> float:
        """Weights, gradients and (ZeRO-1 sharded) optimizer state of ``layers`` layers per GPU."""
        per_gpu_params = (layers * self.layer_params() + extra_params) / tp
        return per_gpu_params * self._bytes_per_param(dp_shard)

    def activation_bytes(self, layers: int, tp: int, sequence_parallel: bool = True) -> float:
        """Stored activations of one in-flight micro-batch over ``layers`` layers per GPU."""
        per_layer = ACTIVATION_BYTES_PER_TOKEN_HIDDEN * self.tokens_per_microbatch * self.hidden
        return layers * per_layer / (tp if sequence_parallel else 1)

    def boundary_bytes(self) -> int:
        """The bf16 hidden state that crosses a pipeline boundary."""
        return 2 * self.tokens_per_microbatch * self.hidden

    @classmethod
    def from_config(cls, cfg, micro_batch_size: int = 1) -> "ModelSpec":
        """From a ``models.config.GPTConfig``."""
        return cls(num_layers=cfg.layers, hidden=cfg.hidden, ffn=cfg.ffn, num_heads=cfg.heads,
                   num_kv_heads=cfg.kv_heads, vocab=cfg.vocab_size, seq_len=cfg.seq_len,
                   micro_batch_size=micro_batch_size)


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
        """Fraction of linear TP scaling kept at degree ``k``: ``1 / (1 + overhead * (k - 1))``."""
        return 1.0 / (1.0 + self.tp_overhead * (k - 1))

    def group_speed(self, tp: int, min_speed: float) -> float:
        """Relative throughput of a TP group: its slowest member sets the pace of all ``tp``."""
        return tp * min_speed * self.tp_efficiency(tp)

    def fwd_layer_time(self, tokens: float, sum_sq: float, tp: int, speed: float) -> float:
        work = self.alpha * tokens + self.beta * sum_sq
        return work / max(self.group_speed(tp, speed), 1e-9)

    def p2p_time(self, nbytes: float, same_node: bool = False) -> float:
        bandwidth = self.intra_node_bandwidth if same_node else self.p2p_bandwidth
        return self.p2p_latency + nbytes / bandwidth

    @classmethod
    def b200(cls, spec: ModelSpec, sustained_tflops: float = 1000.0, attn_tflops: float = 400.0) -> "ModelProfile":
        """Analytic B200 profile.  alpha: the layer's dense matmul FLOPs per token (2 per weight,
        norms excluded) at the sustained GEMM rate; beta: causal attention FLOPs per squared
        token (QK^T and PV over half the score matrix: 2 * heads * head_dim) at the attention
        kernel's rate.  Links: NVLink 5 at the measured ~770 GB/s per direction inside a node,
        400 Gb/s-class NICs between nodes."""
        matmul_flops_per_token = 2 * (spec.layer_params() - 2 * spec.hidden)
        attention_flops_per_sq_token = 2 * spec.num_heads * spec.head_dim
        return cls(alpha=matmul_flops_per_token / (sustained_tflops * 1e12),
                   beta=attention_flops_per_sq_token / (attn_tflops * 1e12),
                   p2p_bandwidth=50e9, intra_node_bandwidth=770e9, p2p_latency=10e-6)

    @classmethod
    def fit(cls, samples: Sequence[tuple[float, float, float]],
            tp_samples: Sequence[tuple[int, float, float]] = (), **fields) -> "ModelProfile":
        """Least-squares profile from measured per-layer forward times.

        ``samples``: ``(tokens, sum_sq, seconds)`` at TP=1 -- fits ``alpha`` and ``beta``
        (non-negative).  ``tp_samples``: ``(k, seconds_at_k, seconds_at_1)`` for the same work --
        fits ``tp_overhead`` from ``t_1 / (k t_k) = 1 / (1 + o (k - 1))``.  Other fields pass
        through ``fields``."""
        import numpy as np

        a = np.array([[n, q] for n, q, _ in samples], dtype=np.float64)
        y = np.array([t for _, _, t in samples], dtype=np.float64)
        if len(samples) < 2 or np.linalg.matrix_rank(a) < 2:
            alpha = float(np.sum(y) / max(np.sum(a[:, 0]), 1e-30)) if len(samples) else 0.0
            beta = 0.0
        else:
            (alpha, beta), *_ = np.linalg.lstsq(a, y, rcond=None)
            if beta < 0:  # attention cannot speed a layer up: refit the token term alone
                alpha, beta = float(a[:, 0] @ y / (a[:, 0] @ a[:, 0])), 0.0
        if tp_samples:
            # (k t_k / t_1) - 1 = o (k - 1): one-parameter least squares through the origin
            xs = np.array([k - 1 for k, _, _ in tp_samples], dtype=np.float64)
            ys = np.array([k * tk / t1 - 1.0 for k, tk, t1 in tp_samples], dtype=np.float64)
            fields.setdefault("tp_overhead", max(0.0, float(xs @ ys / max(xs @ xs, 1e-30))))
        return cls(alpha=float(alpha), beta=float(beta), **fields)

    def to_json(self) -> dict:
        from dataclasses import asdict

        return asdict(self)

    @classmethod
    def calibrated(cls, spec: ModelSpec, directory=None) -> "ModelProfile | None":
        """The measured profile (``bench/profile_gpu.py`` output under ``plan/profiles/``) of a
        model with ``spec``'s layer shape, or None.  Link fields keep the analytic B200 values."""
        import json
        from pathlib import Path

        root = Path(directory) if directory is not None else Path(__file__).resolve().parent / "profiles"
        if not root.is_dir():
            return None
        for path in sorted(root.glob("*.json")):
            doc = json.loads(path.read_text())
            shape = doc.get("shape", {})
            if (shape.get("hidden"), shape.get("ffn"), shape.get("heads"), shape.get("kv_heads")) == (
                    spec.hidden, spec.ffn, spec.num_heads, spec.num_kv_heads):
                analytic = cls.b200(spec)
                measured = {k: v for k, v in doc["profile"].items() if k in ("alpha", "beta", "bwd_ratio",
                                                                             "tp_overhead")}
                from dataclasses import replace

                return replace(analytic, **measured)
        return None

    @classmethod
    def from_json(cls, d: dict) -> "ModelProfile":
        return cls(**d)
