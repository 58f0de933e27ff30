"""Model configurations (architecture shapes) used by the GPU data plane and the planner.

Presets cover the model families named by the benchmark configs: a Llama-3-8B-shaped dense
decoder (GQA + SwiGLU + RoPE), a Mixtral-8x7B-shaped MoE decoder, a GPT-style 1.3B decoder,
and small shapes for tests.  The reference framework's only executable model is an MLP
stack (``resihp/runtime/reference_model.py:32-46``); its GPU models come from Megatron-Core
(``resihp/runtime/megatron_runtime.py``), which this package replaces.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class GPTConfig:
    name: str = "custom"
    vocab_size: int = 32000
    hidden: int = 1024
    layers: int = 4
    heads: int = 16
    kv_heads: int = 16
    ffn: int = 4096
    seq_len: int = 2048
    rope_theta: float = 500000.0
    norm_eps: float = 1e-5
    init_std: float = 0.02
    # mixture of experts (0 = dense)
    num_experts: int = 0
    top_k: int = 2
    moe_every: int = 1
    # MLP: "swiglu" (w1, w3 -> silu(w1 x) * w3 x -> w2) or "gelu" (w1 -> gelu -> w2, the GPT MLP)
    mlp: str = "swiglu"

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def gated(self) -> bool:
        """Gated MLP (SwiGLU: two input projections) or plain (GELU: one)."""
        if self.mlp not in ("swiglu", "gelu"):
            raise ValueError(f"unknown mlp {self.mlp!r}")
        return self.mlp == "swiglu"

    @property
    def mlp_in(self) -> int:
        """Rows of the MLP's input projection (``2 * ffn`` gated, ``ffn`` plain)."""
        return (2 if self.gated else 1) * self.ffn

    @property
    def mlp_mats(self) -> int:
        return 3 if self.gated else 2

    def layer_params(self) -> int:
        H, F = self.hidden, self.ffn
        attn = self.qkv_rows * H + H * self.heads * self.head_dim + 2 * H
        experts = self.num_experts if self.is_moe else 1
        mlp = self.mlp_mats * H * F * experts + (H * self.num_experts if self.is_moe else 0)
        return attn + mlp

    def num_params(self) -> int:
        return self.layers * self.layer_params() + 2 * self.vocab_size * self.hidden + self.hidden

    def flops_per_token(self, seq_len: int | None = None) -> float:
        """Training FLOPs per token: 6 x matmul params + causal attention (fwd + bwd)."""
        S = seq_len or self.seq_len
        H, F = self.hidden, self.ffn
        dense_mm = (self.qkv_rows * H + H * self.heads * self.head_dim
                    + (self.mlp_mats * H * F) * (self.top_k if self.is_moe else 1))
        matmul = self.layers * dense_mm + self.vocab_size * H
        attn = self.layers * 4 * self.heads * self.head_dim * S / 2  # QK^T and PV, causal half, per token
        return 6.0 * matmul + 3.0 * attn

    def to_dict(self) -> dict:
        return asdict(self)

    def with_(self, **kw) -> "GPTConfig":
        return replace(self, **kw)


LLAMA3_8B = GPTConfig(name="llama3-8b", vocab_size=128256, hidden=4096, layers=32, heads=32, kv_heads=8, ffn=14336,
                      seq_len=4096, rope_theta=500000.0)
MIXTRAL_8X7B = GPTConfig(name="mixtral-8x7b", vocab_size=32000, hidden=4096, layers=32, heads=32, kv_heads=8,
                         ffn=14336, seq_len=4096, rope_theta=1000000.0, num_experts=8, top_k=2)
GPT_1P3B = GPTConfig(name="gpt-1.3b", vocab_size=50304, hidden=2048, layers=24, heads=16, kv_heads=16, ffn=8192,
                     seq_len=2048, rope_theta=10000.0, mlp="gelu")
TINY = GPTConfig(name="tiny", vocab_size=512, hidden=256, layers=2, heads=4, kv_heads=2, ffn=512, seq_len=128)

PRESETS = {c.name: c for c in (LLAMA3_8B, MIXTRAL_8X7B, GPT_1P3B, TINY)}


def get_config(name: str, **overrides) -> GPTConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[name].with_(**overrides) if overrides else PRESETS[name]
