// Token cross-entropy over a large vocabulary, fused forward + backward.
//
// One CTA per token row.  Pass 1 computes the row max and the sum of exponentials with an
// online (rescaling) reduction over 16-byte vectors; pass 2 writes the gradient
// (softmax - onehot) * grad_scale over the logits in place (bf16), so the logits buffer
// becomes dlogits without a second allocation.  Rows whose label equals `ignore_index`
// get loss 0 and a zero gradient.  The vocabulary may be a shard [v0, v0 + Vl) of a
// vocab-parallel layer: `lse_out` then holds the local log-sum-exp, and the label logit is
// taken only when the label falls inside the shard.
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100.cuh"

namespace rb {

namespace {

constexpr int kCeThreads = 512;

__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  const float mn = fmaxf(m, m2);
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

template <bool VEC>
__global__ void __launch_bounds__(kCeThreads) ce_kernel(__nv_bfloat16* __restrict__ logits, long long ld,
                                                        const int64_t* __restrict__ labels, float* __restrict__ loss,
                                                        float* __restrict__ lse_out, int V, long long v0,
                                                        float grad_scale, long long ignore_index, int write_grad) {
  __shared__ float sm[32], ss[32];
  __shared__ float s_stat[2];
  const long long row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  const long long label = labels[row];
  const bool ignored = (label == ignore_index);
  const int nv = VEC ? V / 8 : 0;  // rows that are not 16-byte aligned take the scalar path

  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x; c < nv; c += kCeThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + c * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float vals[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      vals[2 * j] = f.x;
      vals[2 * j + 1] = f.y;
    }
    float lm = vals[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, vals[j]);
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ls += __expf(vals[j] - lm);
    merge(m, s, lm, ls);
  }
  for (int c = nv * 8 + threadIdx.x; c < V; c += kCeThreads) merge(m, s, __bfloat162float(x[c]), 1.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[wid] = m;
    ss[wid] = s;
  }
  __syncthreads();
  if (wid == 0) {
    m = (lane < kCeThreads / 32) ? sm[lane] : -INFINITY;
    s = (lane < kCeThreads / 32) ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, m2, s2);
    }
    if (lane == 0) {
      s_stat[0] = m;
      s_stat[1] = s;
    }
  }
  __syncthreads();
  const float rmax = s_stat[0];
  const float rsum = s_stat[1];
  const float lse = rmax + logf(rsum);
  const long long lbl_local = label - v0;
  const bool in_shard = !ignored && lbl_local >= 0 && lbl_local < V;
  if (threadIdx.x == 0) {
    const float xl = in_shard ? __bfloat162float(x[lbl_local]) : 0.f;
    if (lse_out != nullptr) lse_out[row] = lse;
    loss[row] = ignored ? 0.f : (lse - xl);
  }
  if (!write_grad) return;
  __syncthreads();  // thread 0 has read x[label] before it is overwritten
  const float inv = 1.f / rsum;
  const float gs = ignored ? 0.f : grad_scale;
  for (int c = threadIdx.x; c < nv; c += kCeThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(x + c * 8);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      const long long col = static_cast<long long>(c) * 8 + 2 * j;
      float g0 = __expf(f.x - rmax) * inv;
      float g1 = __expf(f.y - rmax) * inv;
      if (in_shard && col == lbl_local) g0 -= 1.f;
      if (in_shard && col + 1 == lbl_local) g1 -= 1.f;
      w[j] = pack_bf16x2(g0 * gs, g1 * gs);
    }
    u.x = w[0]; u.y = w[1]; u.z = w[2]; u.w = w[3];
    *reinterpret_cast<uint4*>(x + c * 8) = u;
  }
  for (int c = nv * 8 + threadIdx.x; c < V; c += kCeThreads) {
    float g = __expf(__bfloat162float(x[c]) - rmax) * inv;
    if (in_shard && c == lbl_local) g -= 1.f;
    x[c] = __float2bfloat16_rn(g * gs);
  }
}

}  // namespace

int cross_entropy_fwd_bwd(void* logits, long long ld, const int64_t* labels, float* loss, float* lse, int T, int V,
                          long long v0, float grad_scale, long long ignore_index, int write_grad, cudaStream_t s) {
  if (T <= 0) return 0;
  const bool vec = !((reinterpret_cast<uintptr_t>(logits) & 15) || (ld % 8));
  if (vec)
    ce_kernel<true><<<T, kCeThreads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld, labels, loss, lse, V, v0,
                                             grad_scale, ignore_index, write_grad);
  else
    ce_kernel<false><<<T, kCeThreads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld, labels, loss, lse, V,
                                              v0, grad_scale, ignore_index, write_grad);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rb
