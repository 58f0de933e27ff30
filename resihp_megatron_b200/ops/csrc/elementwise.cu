// Bandwidth-bound kernels of the decoder: RMSNorm (fwd / bwd), rotary embedding, SwiGLU,
// token embedding gather / deterministic scatter, and the fused Adam update.
//
// All kernels move 16-byte vectors (8 bf16 or 4 fp32) and keep reductions deterministic:
// cross-row sums (RMSNorm weight gradient, embedding gradient) are computed by fixed
// assignments of rows to CTAs and summed in a fixed order, never with float atomics, so a
// result does not depend on scheduling.
#include <cuda_runtime.h>

#include <cstdint>

#include "act_common.cuh"
#include "fp8_common.cuh"
#include "sm100.cuh"

namespace rb {

namespace {

__device__ __forceinline__ void load_bf16x8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = (l < THREADS / 32) ? sh[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) sh[0] = t;
  }
  __syncthreads();
  t = sh[0];
  __syncthreads();
  return t;
}

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 4;  // up to 256 * 4 * 8 = 8192 features per row

// y = x * rsqrt(mean(x^2) + eps) * w ; rstd saved for the backward pass.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   __nv_bfloat16* __restrict__ y,
                                                                   float* __restrict__ rstd, int H, float eps) {
  __shared__ float sh[32];
  const long long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  float v[kNormMaxVec][8];
  float ss = 0.f;
  const int nvec = H / 8;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = (threadIdx.x + i * kNormThreads);
    if (c < nvec) {
      load_bf16x8(xr + c * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum<kNormThreads>(ss, sh);
  const float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd[row] = r;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = (threadIdx.x + i * kNormThreads);
    if (c < nvec) {
      float wv[8];
      load_bf16x8(w + c * 8, wv);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * r * wv[j];
      store_bf16x8(y + row * H + c * 8, o);
    }
  }
}

// RMSNorm straight to block-scaled fp8 (the fp8 projections' input): the same arithmetic as
// rmsnorm_fwd_kernel up to the bf16 output, then each 1 x 128 block of the bf16 row is quantised
// exactly as fp8_quantize would (power-of-two scale from the block's amax, round to nearest even).
// The 16 threads holding one block (16 x 8 consecutive features) reduce its amax with shuffles.
// Scale of block cb of this row: s[cb * s_kb + row * s_row].  One atomicMax per row on `amax`.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fp8_kernel(const __nv_bfloat16* __restrict__ x,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   float* __restrict__ rstd, int H, float eps,
                                                                   int fmt, uint8_t* __restrict__ q, float* s,
                                                                   long long s_kb, long long s_row,
                                                                   unsigned int* amax) {
  __shared__ float sh[32];
  __shared__ uint32_t wmax[kNormThreads / 32];
  const long long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  float v[kNormMaxVec][8];
  float ss = 0.f;
  const int nvec = H / 8;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = (threadIdx.x + i * kNormThreads);
    if (c < nvec) {
      load_bf16x8(xr + c * 8, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum<kNormThreads>(ss, sh);
  const float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0 && rstd != nullptr) rstd[row] = r;
  const int F = fp8_max_exp(fmt);
  uint32_t rmax = 0;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = (threadIdx.x + i * kNormThreads);
    const bool on = c < nvec;  // H % 128 == 0: a block's 16 threads are all on or all off
    float o[8];
    uint32_t m = 0;
    if (on) {
      float wv[8];
      load_bf16x8(w + c * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j] = __bfloat162float(__float2bfloat16_rn(v[i][j] * r * wv[j]));
        m = max(m, __float_as_uint(o[j]) & 0x7fffffffu);
      }
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
    rmax = max(rmax, m);
    if (on) {
      const int e = fp8_scale_exp(m, F);
      const float inv = exp2_int(-e);
      uint2 u;
      u.x = cvt4_fp8(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv, fmt);
      u.y = cvt4_fp8(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv, fmt);
      *reinterpret_cast<uint2*>(q + row * H + c * 8) = u;
      if ((threadIdx.x & 15) == 0) s[static_cast<long long>(c / 16) * s_kb + row * s_row] = exp2_int(e);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) rmax = max(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = rmax;
  __syncthreads();
  if (threadIdx.x == 0 && amax != nullptr) {
    uint32_t m = 0;
    for (int k = 0; k < kNormThreads / 32; ++k) m = max(m, wmax[k]);
    atomicMax(amax, m);
  }
}

// dx = rstd * (w*dy - xhat * mean(xhat * w*dy)) (+ dres) ; per-CTA partial dw over a fixed
// block of ROWS rows written to dw_part[blockIdx.x, :] (fp32), reduced later in order.
constexpr int kNormBwdRows = 32;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dy,
    const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, int T,
    int H) {
  __shared__ float sh[32];
  const int nvec = H / 8;
  float wv[kNormMaxVec][8];
  float dwacc[kNormMaxVec][8];
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
#pragma unroll
    for (int j = 0; j < 8; ++j) dwacc[i][j] = 0.f;
    if (c < nvec) load_bf16x8(w + c * 8, wv[i]);
  }
  const int r0 = blockIdx.x * kNormBwdRows;
  const int r1 = min(T, r0 + kNormBwdRows);
  for (int row = r0; row < r1; ++row) {
    const long long off = static_cast<long long>(row) * H;
    const float r = rstd[row];
    float xh[kNormMaxVec][8], g[kNormMaxVec][8];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormMaxVec; ++i) {
      const int c = threadIdx.x + i * kNormThreads;
      if (c < nvec) {
        load_bf16x8(x + off + c * 8, xh[i]);
        load_bf16x8(dy + off + c * 8, g[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] *= r;
          dwacc[i][j] += g[i][j] * xh[i][j];
          g[i][j] *= wv[i][j];
          dot += g[i][j] * xh[i][j];
        }
      }
    }
    dot = block_sum<kNormThreads>(dot, sh) / H;
#pragma unroll
    for (int i = 0; i < kNormMaxVec; ++i) {
      const int c = threadIdx.x + i * kNormThreads;
      if (c < nvec) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = r * (g[i][j] - xh[i][j] * dot);
        if (dres != nullptr) {
          float d[8];
          load_bf16x8(dres + off + c * 8, d);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += d[j];
        }
        store_bf16x8(dx + off + c * 8, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < nvec) {
      float4* dst = reinterpret_cast<float4*>(dw_part + static_cast<long long>(blockIdx.x) * H + c * 8);
      dst[0] = make_float4(dwacc[i][0], dwacc[i][1], dwacc[i][2], dwacc[i][3]);
      dst[1] = make_float4(dwacc[i][4], dwacc[i][5], dwacc[i][6], dwacc[i][7]);
    }
  }
}

// out[c] (+)= sum_{b < nb} part[b, c], summed in increasing b.
__global__ void colsum_kernel(const float* __restrict__ part, float* __restrict__ out, int nb, int H,
                              int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int b = 0; b < nb; ++b) s += part[static_cast<long long>(b) * H + c];
  out[c] = accumulate ? out[c] + s : s;
}

// Rotary embedding, rotate-half convention, in place on a [T, heads, D] strided view.
// cos/sin tables are [S, D/2] fp32; token t uses position pos0 + (t % S).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ q, long long row_stride, int heads, int D,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t, int S, int T,
                            int inverse) {
  const int half = D / 2;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(T) * heads * (half / 2);
  if (idx >= total) return;
  const int pairs = half / 2;  // two rotation pairs per thread
  const int p = idx % pairs;
  const long long th = idx / pairs;
  const int h = th % heads;
  const int t = th / heads;
  const int pos = t % S;
  __nv_bfloat16* base = q + static_cast<long long>(t) * row_stride + static_cast<long long>(h) * D;
  const int i = 2 * p;
  const float2 lo = unpack_bf16x2(*reinterpret_cast<uint32_t*>(base + i));
  const float2 hi = unpack_bf16x2(*reinterpret_cast<uint32_t*>(base + half + i));
  const float c0 = cos_t[pos * half + i], c1 = cos_t[pos * half + i + 1];
  float s0 = sin_t[pos * half + i], s1 = sin_t[pos * half + i + 1];
  if (inverse) {
    s0 = -s0;
    s1 = -s1;
  }
  // (x1, x2) -> (x1 c - x2 s, x2 c + x1 s)
  *reinterpret_cast<uint32_t*>(base + i) = pack_bf16x2(lo.x * c0 - hi.x * s0, lo.y * c1 - hi.y * s1);
  *reinterpret_cast<uint32_t*>(base + half + i) = pack_bf16x2(hi.x * c0 + lo.x * s0, hi.y * c1 + lo.y * s1);
}


// gu = [T, 2F] with gate in [:, :F] and up in [:, F:]; a = silu(gate) * up.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ a, int T,
                                  int F) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  const int nv = F / 8;
  if (idx >= static_cast<long long>(T) * nv) return;
  const int t = idx / nv, c = idx % nv;
  float g[8], u[8], o[8];
  load_bf16x8(gu + static_cast<long long>(t) * 2 * F + c * 8, g);
  load_bf16x8(gu + static_cast<long long>(t) * 2 * F + F + c * 8, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * u[j];
  store_bf16x8(a + static_cast<long long>(t) * F + c * 8, o);
}

// dgu[:, :F] = da * up * silu'(gate) ; dgu[:, F:] = da * silu(gate).  May run in place (dgu == gu).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* gu, const __nv_bfloat16* __restrict__ da,
                                  __nv_bfloat16* dgu, int T, int F) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  const int nv = F / 8;
  if (idx >= static_cast<long long>(T) * nv) return;
  const int t = idx / nv, c = idx % nv;
  const long long gofs = static_cast<long long>(t) * 2 * F + c * 8;
  float g[8], u[8], d[8], dg[8], du[8];
  load_bf16x8(gu + gofs, g);
  load_bf16x8(gu + gofs + F, u);
  load_bf16x8(da + static_cast<long long>(t) * F + c * 8, d);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sg = 1.f / (1.f + __expf(-g[j]));
    const float s = g[j] * sg;
    du[j] = d[j] * s;
    dg[j] = d[j] * u[j] * (sg * (1.f + g[j] * (1.f - sg)));
  }
  store_bf16x8(dgu + gofs, dg);
  store_bf16x8(dgu + gofs + F, du);
}

// GELU (act_common.cuh), elementwise over [n] (n % 8 == 0).

__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ a, long long n8) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float x[8], o[8];
  load_bf16x8(h + i * 8, x);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = gelu_tanh(x[j]);
  store_bf16x8(a + i * 8, o);
}

// dh = da * gelu'(h).  May run in place (dh == h).
__global__ void gelu_bwd_kernel(const __nv_bfloat16* h, const __nv_bfloat16* __restrict__ da, __nv_bfloat16* dh,
                                long long n8) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float x[8], d[8], o[8];
  load_bf16x8(h + i * 8, x);
  load_bf16x8(da + i * 8, d);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x2 = x[j] * x[j];
    const float t = tanhf(kGeluC * (x[j] + kGeluA * x2 * x[j]));
    const float dg = 0.5f * (1.f + t) + 0.5f * x[j] * (1.f - t * t) * kGeluC * (1.f + 3.f * kGeluA * x2);
    o[j] = d[j] * dg;
  }
  store_bf16x8(dh + i * 8, o);
}

// Delayed-scaling history update, one thread per recorded tensor: hist[i] = [pending[i],
// hist[i][0 .. len-2]] and pending[i] = 0.
__global__ void amax_history_push_kernel(float* __restrict__ hist, float* __restrict__ pending, int n, int len) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float* h = hist + static_cast<long long>(i) * len;
  for (int j = len - 1; j > 0; --j) h[j] = h[j - 1];
  h[0] = pending[i];
  pending[i] = 0.f;
}

// The MLP activation written straight as block-scaled fp8 (the fc2 input): GELU of h [T, F]
// (GATED = false) or silu(gate) * up of gu [T, 2F] (GATED = true), rounded to bf16 exactly as
// gelu_fwd_kernel / swiglu_fwd_kernel round it, then each 1 x 128 block of a row quantised as
// fp8_quantize would.  Thread i covers features [8 i, 8 i + 8) of the flattened [T, F] output,
// so the 16 consecutive threads of a block (F % 128 == 0) reduce its amax with shuffles.  Scale
// of block cb of row t: s[cb * s_kb + t * s_row].  One atomicMax per CTA on `amax`.
template <bool GATED>
__global__ void __launch_bounds__(256) act_fp8_kernel(const __nv_bfloat16* __restrict__ in, int T, int F, int fmt,
                                                      uint8_t* __restrict__ q, float* __restrict__ s, long long s_kb,
                                                      long long s_row, unsigned int* amax) {
  __shared__ uint32_t wmax[8];
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nv = F / 8;
  const bool on = i < static_cast<long long>(T) * nv;  // whole 16-thread groups (T * nv % 16 == 0)
  const long long t = on ? i / nv : 0;
  const int c = on ? static_cast<int>(i % nv) : 0;
  float o[8];
  uint32_t m = 0;
  if (on) {
    if (GATED) {
      float g[8], u[8];
      load_bf16x8(in + t * 2 * F + c * 8, g);
      load_bf16x8(in + t * 2 * F + F + c * 8, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __bfloat162float(__float2bfloat16_rn(silu(g[j]) * u[j]));
    } else {
      float x[8];
      load_bf16x8(in + t * F + c * 8, x);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = __bfloat162float(__float2bfloat16_rn(gelu_tanh(x[j])));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) m = max(m, __float_as_uint(o[j]) & 0x7fffffffu);
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (on) {
    const int e = fp8_scale_exp(m, fp8_max_exp(fmt));
    const float inv = exp2_int(-e);
    uint2 u;
    u.x = cvt4_fp8(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv, fmt);
    u.y = cvt4_fp8(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv, fmt);
    *reinterpret_cast<uint2*>(q + t * F + c * 8) = u;
    if ((threadIdx.x & 15) == 0) s[static_cast<long long>(c / 16) * s_kb + t * s_row] = exp2_int(e);
  }
  uint32_t bm = m;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) bm = max(bm, __shfl_xor_sync(0xffffffffu, bm, off));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = bm;
  __syncthreads();
  if (threadIdx.x == 0 && amax != nullptr) {
    uint32_t mm = 0;
    for (int k = 0; k < 8; ++k) mm = max(mm, wmax[k]);
    atomicMax(amax, mm);
  }
}

// x[t, :] = E[ids[t], :]
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ E,
                                     __nv_bfloat16* __restrict__ x, int T, int H, int V, int* err) {
  const int t = blockIdx.x;
  long long id = ids[t];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) record_error(err, kErrBadArg);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(E + id * H);
  uint4* dst = reinterpret_cast<uint4*>(x + static_cast<long long>(t) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

// Embedding backward on the ids sorted stably by value (`vals`, with original positions
// `order`): block i owns position i; if it starts a run of equal ids it sums that run's rows of dx
// in position order and adds them to dE[id, :] (fixed order: deterministic), else it returns.  No
// data-dependent sizes reach the host, so the whole backward can be captured in a CUDA graph.
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ vals, const int64_t* __restrict__ order, int T,
                                     const __nv_bfloat16* __restrict__ dx, float* __restrict__ dE, int H) {
  const int i = blockIdx.x;
  const long long id = vals[i];
  if (i > 0 && vals[i - 1] == id) return;
  int end = i + 1;
  while (end < T && vals[end] == id) ++end;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = i; s < end; ++s) {
      float v[8];
      load_bf16x8(dx + order[s] * H + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    float4* dst = reinterpret_cast<float4*>(dE + id * H + c);
    float4 a = dst[0], b = dst[1];
    a.x += acc[0]; a.y += acc[1]; a.z += acc[2]; a.w += acc[3];
    b.x += acc[4]; b.y += acc[5]; b.z += acc[6]; b.w += acc[7];
    dst[0] = a;
    dst[1] = b;
  }
}

// Adam(W) on flat fp32 master weights, with the gradient scale (e.g. 1 / global tokens) and
// the bf16 model copy fused in.  Formula order follows torch.optim.Adam (single tensor):
//   g = grad * scale (+ wd * p for classic L2) ; m = lerp(m, g, 1-b1) ; v = b2 v + (1-b2) g^2
//   p -= lr / bc1 * m / (sqrt(v) / sqrt(bc2) + eps)
__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ grad, float* __restrict__ m,
                            float* __restrict__ v, __nv_bfloat16* __restrict__ p_bf16, long long n, float lr,
                            float b1, float b2, float eps, float wd, int decoupled, float bc1, float bc2_sqrt,
                            float grad_scale, int zero_grad, const float* __restrict__ bc_dev) {
  const long long i4 = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i4 >= n) return;
  if (bc_dev != nullptr) {  // bias corrections of this step from device memory (replayed CUDA graphs)
    bc1 = bc_dev[0];
    bc2_sqrt = bc_dev[1];
  }
  const float step_size = lr / bc1;
  const int cnt = (n - i4) >= 4 ? 4 : static_cast<int>(n - i4);
  float pp[4], gg[4], mm[4], vv[4];
  if (cnt == 4) {
    *reinterpret_cast<float4*>(pp) = *reinterpret_cast<const float4*>(p + i4);
    *reinterpret_cast<float4*>(gg) = *reinterpret_cast<const float4*>(grad + i4);
    *reinterpret_cast<float4*>(mm) = *reinterpret_cast<const float4*>(m + i4);
    *reinterpret_cast<float4*>(vv) = *reinterpret_cast<const float4*>(v + i4);
  } else {
    for (int j = 0; j < cnt; ++j) {
      pp[j] = p[i4 + j]; gg[j] = grad[i4 + j]; mm[j] = m[i4 + j]; vv[j] = v[i4 + j];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float g = gg[j] * grad_scale;
    if (wd != 0.f) {
      if (decoupled) pp[j] *= (1.f - lr * wd);
      else g = g + wd * pp[j];
    }
    mm[j] = mm[j] + (1.f - b1) * (g - mm[j]);
    vv[j] = vv[j] * b2 + (1.f - b2) * g * g;
    const float denom = sqrtf(vv[j]) / bc2_sqrt + eps;
    pp[j] = pp[j] - step_size * (mm[j] / denom);
  }
  if (cnt == 4) {
    *reinterpret_cast<float4*>(p + i4) = *reinterpret_cast<float4*>(pp);
    *reinterpret_cast<float4*>(m + i4) = *reinterpret_cast<float4*>(mm);
    *reinterpret_cast<float4*>(v + i4) = *reinterpret_cast<float4*>(vv);
    if (zero_grad) *reinterpret_cast<float4*>(const_cast<float*>(grad) + i4) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p_bf16 != nullptr) {
      uint2 u;
      u.x = pack_bf16x2(pp[0], pp[1]);
      u.y = pack_bf16x2(pp[2], pp[3]);
      *reinterpret_cast<uint2*>(p_bf16 + i4) = u;
    }
  } else {
    for (int j = 0; j < cnt; ++j) {
      p[i4 + j] = pp[j]; m[i4 + j] = mm[j]; v[i4 + j] = vv[j];
      if (zero_grad) const_cast<float*>(grad)[i4 + j] = 0.f;
      if (p_bf16 != nullptr) p_bf16[i4 + j] = __float2bfloat16_rn(pp[j]);
    }
  }
}

// Sum of squares of a flat fp32 buffer into per-CTA partials (fixed grid -> deterministic).
__global__ void sumsq_partial_kernel(const float* __restrict__ x, long long n, float* __restrict__ part) {
  __shared__ float sh[32];
  float s = 0.f;
  for (long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x * 4) {
    if (i + 4 <= n) {
      const float4 v = *reinterpret_cast<const float4*>(x + i);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    } else {
      for (long long j = i; j < n; ++j) s += x[j] * x[j];
    }
  }
  s = block_sum<256>(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

}  // namespace

static inline int cdiv_ll(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

int rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int T, int H, float eps, cudaStream_t s) {
  if (H % 8 || H > kNormThreads * kNormMaxVec * 8) return -1;
  rmsnorm_fwd_kernel<<<T, kNormThreads, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                                reinterpret_cast<const __nv_bfloat16*>(w),
                                                reinterpret_cast<__nv_bfloat16*>(y), rstd, H, eps);
  return static_cast<int>(cudaGetLastError());
}

int rmsnorm_fp8(const void* x, const void* w, float* rstd, int T, int H, float eps, int fmt, void* q, float* s,
                long long s_kb, long long s_row, unsigned int* amax, cudaStream_t st) {
  if (H % 128 || H > kNormThreads * kNormMaxVec * 8 || (fmt != kFp8E4M3 && fmt != kFp8E5M2)) return -1;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 7) || s == nullptr) return -2;
  if (T == 0) return 0;
  rmsnorm_fp8_kernel<<<T, kNormThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                                 reinterpret_cast<const __nv_bfloat16*>(w), rstd, H, eps, fmt,
                                                 static_cast<uint8_t*>(q), s, s_kb, s_row, amax);
  return static_cast<int>(cudaGetLastError());
}

int act_fp8(const void* in, int gated, int T, int F, int fmt, void* q, float* s, long long s_kb, long long s_row,
            unsigned int* amax, cudaStream_t st) {
  if (F % 128 || T < 0 || (fmt != kFp8E4M3 && fmt != kFp8E5M2)) return -1;
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(q) & 7) || s == nullptr) return -2;
  if (T == 0) return 0;
  const long long n = static_cast<long long>(T) * (F / 8);
  if (gated)
    act_fp8_kernel<true><<<cdiv_ll(n, 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(in), T, F, fmt,
                                                            static_cast<uint8_t*>(q), s, s_kb, s_row, amax);
  else
    act_fp8_kernel<false><<<cdiv_ll(n, 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(in), T, F, fmt,
                                                             static_cast<uint8_t*>(q), s, s_kb, s_row, amax);
  return static_cast<int>(cudaGetLastError());
}

int rmsnorm_bwd_blocks(int T) { return (T + kNormBwdRows - 1) / kNormBwdRows; }

int rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres, void* dx,
                float* dw, int accumulate, float* part, int T, int H, cudaStream_t s) {
  if (H % 8 || H > kNormThreads * kNormMaxVec * 8) return -1;
  const int nb = rmsnorm_bwd_blocks(T);
  rmsnorm_bwd_kernel<<<nb, kNormThreads, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w), rstd,
      reinterpret_cast<const __nv_bfloat16*>(dy), reinterpret_cast<const __nv_bfloat16*>(dres),
      reinterpret_cast<__nv_bfloat16*>(dx), part, T, H);
  colsum_kernel<<<cdiv_ll(H, 256), 256, 0, s>>>(part, dw, nb, H, accumulate);
  return static_cast<int>(cudaGetLastError());
}

int rope_apply(void* q, long long row_stride, int heads, int D, const float* cos_t, const float* sin_t, int S,
               int T, int inverse, cudaStream_t s) {
  if (D % 4) return -1;
  const long long total = static_cast<long long>(T) * heads * (D / 4);
  rope_kernel<<<cdiv_ll(total, 256), 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(q), row_stride, heads, D,
                                                   cos_t, sin_t, S, T, inverse);
  return static_cast<int>(cudaGetLastError());
}

int swiglu_fwd(const void* gu, void* a, int T, int F, cudaStream_t s) {
  if (F % 8) return -1;
  const long long total = static_cast<long long>(T) * (F / 8);
  swiglu_fwd_kernel<<<cdiv_ll(total, 256), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(gu),
                                                        reinterpret_cast<__nv_bfloat16*>(a), T, F);
  return static_cast<int>(cudaGetLastError());
}

int swiglu_bwd(const void* gu, const void* da, void* dgu, int T, int F, cudaStream_t s) {
  if (F % 8) return -1;
  const long long total = static_cast<long long>(T) * (F / 8);
  swiglu_bwd_kernel<<<cdiv_ll(total, 256), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(gu),
                                                        reinterpret_cast<const __nv_bfloat16*>(da),
                                                        reinterpret_cast<__nv_bfloat16*>(dgu), T, F);
  return static_cast<int>(cudaGetLastError());
}

int gelu_fwd(const void* h, void* a, long long n, cudaStream_t s) {
  if (n % 8) return -1;
  if (n == 0) return 0;
  gelu_fwd_kernel<<<cdiv_ll(n / 8, 256), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(h),
                                                      reinterpret_cast<__nv_bfloat16*>(a), n / 8);
  return static_cast<int>(cudaGetLastError());
}

int gelu_bwd(const void* h, const void* da, void* dh, long long n, cudaStream_t s) {
  if (n % 8) return -1;
  if (n == 0) return 0;
  gelu_bwd_kernel<<<cdiv_ll(n / 8, 256), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(h),
                                                      reinterpret_cast<const __nv_bfloat16*>(da),
                                                      reinterpret_cast<__nv_bfloat16*>(dh), n / 8);
  return static_cast<int>(cudaGetLastError());
}

int amax_history_push(float* hist, float* pending, int n, int len, cudaStream_t s) {
  if (n < 0 || len < 1) return -1;
  if (n == 0) return 0;
  amax_history_push_kernel<<<(n + 127) / 128, 128, 0, s>>>(hist, pending, n, len);
  return static_cast<int>(cudaGetLastError());
}

int embedding_fwd(const int64_t* ids, const void* E, void* x, int T, int H, int V, int* err, cudaStream_t s) {
  if (H % 8) return -1;
  embedding_fwd_kernel<<<T, 128, 0, s>>>(ids, reinterpret_cast<const __nv_bfloat16*>(E),
                                         reinterpret_cast<__nv_bfloat16*>(x), T, H, V, err);
  return static_cast<int>(cudaGetLastError());
}

int embedding_bwd(const int64_t* vals, const int64_t* order, int T, const void* dx, float* dE, int H,
                  cudaStream_t s) {
  if (H % 8 || T < 0) return -1;
  if (T == 0) return 0;
  embedding_bwd_kernel<<<T, 128, 0, s>>>(vals, order, T, reinterpret_cast<const __nv_bfloat16*>(dx), dE, H);
  return static_cast<int>(cudaGetLastError());
}

int adam_step(float* p, float* grad, float* m, float* v, void* p_bf16, long long n, float lr, float b1, float b2,
              float eps, float wd, int decoupled, float bc1, float bc2_sqrt, float grad_scale, int zero_grad,
              cudaStream_t s, const float* bc_dev) {
  if (n <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(grad) | reinterpret_cast<uintptr_t>(m) |
       reinterpret_cast<uintptr_t>(v)) & 15)
    return -1;
  if (p_bf16 != nullptr && (reinterpret_cast<uintptr_t>(p_bf16) & 7)) return -1;
  const long long nthreads = (n + 3) / 4;
  adam_kernel<<<cdiv_ll(nthreads, 256), 256, 0, s>>>(p, grad, m, v, reinterpret_cast<__nv_bfloat16*>(p_bf16), n,
                                                     lr, b1, b2, eps, wd, decoupled, bc1, bc2_sqrt, grad_scale,
                                                     zero_grad, bc_dev);
  return static_cast<int>(cudaGetLastError());
}

int sumsq_partial(const float* x, long long n, float* part, int nblocks, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(x) & 15) return -1;
  sumsq_partial_kernel<<<nblocks, 256, 0, s>>>(x, n, part);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rb
