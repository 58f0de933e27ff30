// Power-of-two block scales and fp8 conversion shared by the fp8 kernels (quantiser, fused
// RMSNorm -> fp8).  Kept in one place so every producer of fp8 operands rounds identically.
#pragma once

#include <cuda_fp8.h>

#include <cstdint>

namespace rb {

constexpr int kFp8E4M3 = 0;
constexpr int kFp8E5M2 = 1;

// Largest finite value of the format = 1.75 * 2^F.
__host__ __device__ constexpr int fp8_max_exp(int fmt) { return fmt == kFp8E4M3 ? 8 : 15; }

// Exponent e of the power-of-two scale: the smallest e with amax * 2^-e <= 1.75 * 2^F, clamped
// to [-126, 126] so that 2^e and 2^-e are normal floats.  `amax_bits` is the bit pattern of a
// non-negative float; zero, inf and NaN blocks get e = 0.
__device__ __forceinline__ int fp8_scale_exp(uint32_t amax_bits, int F) {
  const int E = static_cast<int>(amax_bits >> 23);
  if (amax_bits == 0 || E == 255) return 0;
  const uint32_t mant = amax_bits & 0x7fffffu;
  int e = (E - 127) - F + (mant > 0x600000u ? 1 : 0);  // 1.75 = 1 + 0x600000 / 2^23
  e = e < -126 ? -126 : (e > 126 ? 126 : e);
  return e;
}

__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

__device__ __forceinline__ uint32_t cvt4_fp8(float a, float b, float c, float d, int fmt) {
  const __nv_fp8_interpretation_t kind = fmt == kFp8E4M3 ? __NV_E4M3 : __NV_E5M2;
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, kind);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, kind);
  return (lo & 0xffffu) | (hi << 16);
}

}  // namespace rb
