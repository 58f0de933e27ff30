// exp2 on the FMA pipe for the attention softmax kernels (attention_sm100.cu,
// attention_bwd_sm100.cu).  A tcgen05 128 x 128 x 128 MMA pair and the 16384 exponentials of its
// probabilities take about the same time on an SM (MUFU: 16 exp2 per clock), so a softmax that
// runs every exp2 on MUFU is the bottleneck; evaluating a fixed share on the FMA pipe with a
// polynomial relieves it.
#pragma once

#include <cuda_runtime.h>

namespace rb {

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for x <= 8 (scores minus a running max that lags the true max by at most
// 2^8).  Range reduction: n = floor(x) from one add in round-down mode against 1.5 * 2^23 (whose
// ulp is 1, so the integer lands in the low mantissa bits), f = x - n in [0, 1) exactly.  2^f is a
// degree-3 polynomial with p(0) = 1 whose coefficients minimise the maximum relative error on
// [0, 1) (Chebyshev / minimax fit by linear programming over 4001 points): 8.6e-5, far below the
// 2^-9 half-ulp of the bf16 P it feeds.  2^n is added to the exponent field.  x <= -127 returns
// +0 (a masked score is -inf).
__device__ __forceinline__ float ex2_fma(float x) {
  constexpr float kC1 = 0.6951168179512024f, kC2 = 0.22764486074447632f, kC3 = 0.07706713676452637f;
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x = fmaxf(x, -127.0f);
  float j;
  asm("add.rm.f32 %0, %1, %2;" : "=f"(j) : "f"(x), "f"(kShift));
  const float f = x - (j - kShift);
  const float poly = fmaf(fmaf(fmaf(kC3, f, kC2), f, kC1), f, 1.0f);
  const int n = __float_as_int(j) - __float_as_int(kShift);
  return __int_as_float(__float_as_int(poly) + (n << 23));
}

// Column c of a score row: of every 8 consecutive columns the first kFma use ex2_fma.
template <int kFma>
__device__ __forceinline__ float ex2_mixed(float x, int c) {
  return (c & 7) < kFma ? ex2_fma(x) : ex2_mufu(x);
}

}  // namespace rb
