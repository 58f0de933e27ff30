// MLP activations shared by the bf16 kernels and the fp8 producers, so every path computes them
// with the same arithmetic (the fp8 operands are then bit-identical to quantising the bf16 ones).
#pragma once

namespace rb {

__device__ __forceinline__ float silu(float g) { return g / (1.f + __expf(-g)); }

// GELU, tanh form (the GPT MLP activation): gelu(h) = 0.5 h (1 + tanh(c (h + 0.044715 h^3))),
// c = sqrt(2 / pi).
constexpr float kGeluC = 0.7978845608028654f;
constexpr float kGeluA = 0.044715f;

__device__ __forceinline__ float gelu_tanh(float x) {
  return 0.5f * x * (1.f + tanhf(kGeluC * (x + kGeluA * x * x * x)));
}

}  // namespace rb
