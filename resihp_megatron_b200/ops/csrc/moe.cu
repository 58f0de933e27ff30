// Mixture-of-experts data path for expert parallelism over NVLink peer memory.
//
//   route      one warp per token: logits = x W_r^T (E <= 16), top-k on logits + bias (the bias
//              only selects), gates = softmax over the selected logits.
//   positions  one CTA: for every (token, slot) its rank among the earlier (token, slot) pairs
//              routed to the same expert, and the per-expert counts -- a fixed-order scan, so the
//              rows an expert sees (and therefore the weight-gradient sums) are deterministic.
//   dispatch   one warp per (token, slot): copy the token row into the holder's receive buffer at
//              its final row (expert-major, then source rank, then position) with 16-byte peer
//              stores; the row index is remembered for the way back.
//   combine    one warp per token: out = residual + sum_k gate_k * y_k with the expert outputs
//              y_k read from the holders' memory (16-byte peer loads, fixed slot order); y_k is
//              kept for the backward.
//   grad push  one warp per (token, slot): dy_k = gate_k * dout to the holder's receive row,
//              dgate_k = <dout, y_k>.
//   grad pull  one warp per token: the router logit gradient of the softmax over the selected
//              logits dl, and dx = dout + sum_k dx_k (from the holders) + dl W_r (the router path).
//   router wgrad  dW_r += dl^T x in two fixed-order passes (token chunks, then their sum).
// Replaces the reference's counts all-to-all + autograd all_to_all_single + index_add
// (resihp/runtime/moe.py:149-265, call sites C11/C12).  Only plain loads and stores touch peer
// memory; the expert GEMMs read only local buffers.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "sm100.cuh"

namespace rb {

namespace {

constexpr int kMaxE = 16;
constexpr int kMaxK = 4;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x [T, H] bf16, w [E, H] bf16, bias [E] fp32 (may be null); H % 256 == 0.
__global__ void moe_route_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                 const float* __restrict__ bias, int T, int H, int E, int k,
                                 float* __restrict__ logits, int* __restrict__ topi, float* __restrict__ gates) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float acc[kMaxE];
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) acc[e] = 0.f;
  const __nv_bfloat16* xr = x + static_cast<long long>(t) * H;
  for (int h = lane * 8; h < H; h += 256) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + h);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) {
      if (e >= E) break;
      const uint4 wv = *reinterpret_cast<const uint4*>(w + static_cast<long long>(e) * H + h);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack_bf16x2(xw[j]), b = unpack_bf16x2(ww[j]);
        acc[e] += a.x * b.x + a.y * b.y;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < kMaxE; ++e)
    if (e < E) acc[e] = warp_sum(acc[e]);
  if (lane != 0) return;
  int sel[kMaxK];
  for (int i = 0; i < k; ++i) {
    int best = -1;
    float bv = -INFINITY;
    for (int e = 0; e < E; ++e) {
      bool used = false;
      for (int j = 0; j < i; ++j) used |= sel[j] == e;
      const float v = acc[e] + (bias != nullptr ? bias[e] : 0.f);
      if (!used && (best < 0 || v > bv)) {
        best = e;
        bv = v;
      }
    }
    sel[i] = best;
  }
  float mx = -INFINITY;
  for (int i = 0; i < k; ++i) mx = fmaxf(mx, acc[sel[i]]);
  float den = 0.f, ex[kMaxK];
  for (int i = 0; i < k; ++i) {
    ex[i] = __expf(acc[sel[i]] - mx);
    den += ex[i];
  }
  for (int e = 0; e < E; ++e) logits[static_cast<long long>(t) * E + e] = acc[e];
  for (int i = 0; i < k; ++i) {
    topi[t * k + i] = sel[i];
    gates[t * k + i] = ex[i] / den;
  }
}

// One CTA of 512 threads: pos[i] for the n = T * k (token, slot) entries in order, counts[e].
constexpr int kPosThreads = 512;
__global__ void __launch_bounds__(kPosThreads) moe_positions_kernel(const int* __restrict__ topi, int n, int E,
                                                                     int* __restrict__ pos, int* __restrict__ counts) {
  __shared__ int part[kMaxE][kPosThreads];
  const int tid = threadIdx.x;
  const int per = (n + kPosThreads - 1) / kPosThreads;
  const int lo = tid * per, hi = min(n, lo + per);
  int c[kMaxE];
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) c[e] = 0;
  for (int i = lo; i < hi; ++i) {
    const int e = topi[i];
#pragma unroll
    for (int q = 0; q < kMaxE; ++q) c[q] += (q == e);
  }
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) part[e][tid] = c[e];
  __syncthreads();
  // exclusive scan over threads, one expert per warp (E <= 16 warps)
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < E) {
    int running = 0;
    for (int base = 0; base < kPosThreads; base += 32) {
      const int v = part[warp][base + lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      part[warp][base + lane] = running + incl - v;
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) counts[warp] = running;
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) c[e] = part[e][tid];
  for (int i = lo; i < hi; ++i) {
    const int e = topi[i];
    int p = 0;
#pragma unroll
    for (int q = 0; q < kMaxE; ++q)
      if (q == e) p = c[q]++;
    pos[i] = p;
  }
}

// An expert may have several holders (replicas); the (token, slot) pairs of expert e are dealt to
// them in a fixed cycle: position p (the pair's rank among this source's pairs of e) goes to
// cycle[e][p % period[e]] -- a speed-weighted round robin whose pattern repeats every period.
constexpr int kMaxPeriod = 64;

struct MoeRoutes {
  int world, me, E, k;
  const int* period;          // [E] cycle length (1: a single holder)
  const int* cycle;           // [E][kMaxPeriod] holder rank of cycle slot j
  const int* cycle_rank;      // [E][kMaxPeriod] rank of slot j among the slots with the same holder
  const int* per_cycle;       // [E][kMaxE] slots of holder h in one cycle
  const long long* rowbase;   // [E][kMaxE] first receive row of (expert e, source me) at holder h
  void* peers[kMaxE];         // receive buffers of every rank ([rows, H] bf16)
};

__global__ void moe_dispatch_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ topi,
                                    const int* __restrict__ pos, int n, int k, int H, MoeRoutes r,
                                    long long* __restrict__ route_row) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int t = i / k, e = topi[i];
  const int p = pos[i], L = r.period[e];
  const int j = p % L;
  const int h = r.cycle[e * kMaxPeriod + j];
  const long long row = r.rowbase[e * kMaxE + h] + static_cast<long long>(p / L) * r.per_cycle[e * kMaxE + h] +
                        r.cycle_rank[e * kMaxPeriod + j];
  if (lane == 0) route_row[i] = row * kMaxE + h;  // holder packed into the row index
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * H);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(r.peers[h]) + row * H);
  for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
}

// out[t] = residual[t] + sum_k gate[t, k] * y_k ; y_k also stored to ycache[t * k + k'].
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ residual, const float* __restrict__ gates,
                                   const long long* __restrict__ route_row, int T, int k, int H, MoeRoutes r,
                                   __nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ ycache) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int j = lane; j < H / 8; j += 32) {
    float acc[8];
    const uint4 rv = reinterpret_cast<const uint4*>(residual + static_cast<long long>(t) * H)[j];
    const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(rw[q]);
      acc[2 * q] = f.x;
      acc[2 * q + 1] = f.y;
    }
    float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < k; ++s) {
      const long long packed = route_row[t * k + s];
      const int h = static_cast<int>(packed % kMaxE);
      const long long row = packed / kMaxE;
      const uint4 yv = __ldcv(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(r.peers[h]) + row * H) + j);
      reinterpret_cast<uint4*>(ycache + (static_cast<long long>(t) * k + s) * H)[j] = yv;
      const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
      const float g = gates[t * k + s];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(yw[q]);
        part[2 * q] += g * f.x;
        part[2 * q + 1] += g * f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0] + part[0], acc[1] + part[1]);
    o.y = pack_bf16x2(acc[2] + part[2], acc[3] + part[3]);
    o.z = pack_bf16x2(acc[4] + part[4], acc[5] + part[5]);
    o.w = pack_bf16x2(acc[6] + part[6], acc[7] + part[7]);
    reinterpret_cast<uint4*>(out + static_cast<long long>(t) * H)[j] = o;
  }
}

// Backward of the combine: dy_k = gate_k * dout pushed to the holder's row; dgate_k = <dout, y_k>.
__global__ void moe_grad_push_kernel(const __nv_bfloat16* __restrict__ dout, const float* __restrict__ gates,
                                     const __nv_bfloat16* __restrict__ ycache, const long long* __restrict__ route_row,
                                     int n, int k, int H, MoeRoutes r, float* __restrict__ dgate) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int t = i / k;
  const long long packed = route_row[i];
  const int h = static_cast<int>(packed % kMaxE);
  const long long row = packed / kMaxE;
  const float g = gates[i];
  float dot = 0.f;
  const uint4* d = reinterpret_cast<const uint4*>(dout + static_cast<long long>(t) * H);
  const uint4* y = reinterpret_cast<const uint4*>(ycache + static_cast<long long>(i) * H);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(r.peers[h]) + row * H);
  for (int j = lane; j < H / 8; j += 32) {
    const uint4 dv = d[j], yv = y[j];
    const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w}, yw[4] = {yv.x, yv.y, yv.z, yv.w};
    uint32_t ow[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = unpack_bf16x2(dw[q]), b = unpack_bf16x2(yw[q]);
      dot += a.x * b.x + a.y * b.y;
      ow[q] = pack_bf16x2(g * a.x, g * a.y);
    }
    dst[j] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
  dot = warp_sum(dot);
  if (lane == 0) dgate[i] = dot;
}

// dx[t] = dout[t] + sum_k dx_k (read from the holders); dlogits[t, e] of the selected-softmax.
__global__ void moe_grad_pull_kernel(const __nv_bfloat16* __restrict__ dout, const float* __restrict__ gates,
                                     const float* __restrict__ dgate, const int* __restrict__ topi,
                                     const long long* __restrict__ route_row, int T, int k, int H, int E, MoeRoutes r,
                                     const __nv_bfloat16* __restrict__ router_w, __nv_bfloat16* __restrict__ dx,
                                     float* __restrict__ dlogits) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  // router logit gradient of the softmax over the selected logits (every lane holds it):
  // gates = softmax(l_sel) -> dl_sel_i = g_i (dgate_i - sum_j g_j dgate_j); zero elsewhere
  float s = 0.f;
  for (int i = 0; i < k; ++i) s += gates[t * k + i] * dgate[t * k + i];
  float dl[kMaxE];
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) dl[e] = 0.f;
  for (int i = 0; i < k; ++i) {
    const int sel = topi[t * k + i];
    const float v = gates[t * k + i] * (dgate[t * k + i] - s);
#pragma unroll
    for (int e = 0; e < kMaxE; ++e)
      if (e == sel) dl[e] = v;
  }
  for (int j = lane; j < H / 8; j += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (dout != nullptr) {  // the residual path, when the experts' input is the residual stream
      const uint4 dv = reinterpret_cast<const uint4*>(dout + static_cast<long long>(t) * H)[j];
      const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(dw[q]);
        acc[2 * q] = f.x;
        acc[2 * q + 1] = f.y;
      }
    }
    for (int s = 0; s < k; ++s) {
      const long long packed = route_row[t * k + s];
      const int h = static_cast<int>(packed % kMaxE);
      const long long row = packed / kMaxE;
      const uint4 v = __ldcv(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(r.peers[h]) + row * H) + j);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(w[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    if (router_w != nullptr) {  // the router path: dx += dl W_r (experts in a fixed order)
#pragma unroll
      for (int e = 0; e < kMaxE; ++e) {
        if (e >= E) break;
        const uint4 wv = reinterpret_cast<const uint4*>(router_w + static_cast<long long>(e) * H)[j];
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(ww[q]);
          acc[2 * q] = fmaf(dl[e], f.x, acc[2 * q]);
          acc[2 * q + 1] = fmaf(dl[e], f.y, acc[2 * q + 1]);
        }
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(dx + static_cast<long long>(t) * H)[j] = o;
  }
  if (lane == 0) {
#pragma unroll
    for (int e = 0; e < kMaxE; ++e)
      if (e < E) dlogits[static_cast<long long>(t) * E + e] = dl[e];
  }
}

// Router weight gradient, deterministic in two passes.  Pass 1: CTA (column block cb, token
// chunk c) sums dl[t, e] * x[t, h] over its chunk's tokens in order for 256 columns (one per
// thread) and every expert, into partial[c][e][h].  Pass 2: one thread per (e, h) adds the chunks'
// partials in chunk order to the fp32 gradient.
constexpr int kRwCols = 256;
constexpr int kRwChunk = 256;

__global__ void __launch_bounds__(kRwCols) moe_router_wgrad_kernel(const float* __restrict__ dlogits,
                                                                    const __nv_bfloat16* __restrict__ x, int T, int H,
                                                                    int E, float* __restrict__ partial) {
  const int h = blockIdx.x * kRwCols + threadIdx.x;
  const int c = blockIdx.y;
  __shared__ float sdl[kRwChunk * kMaxE];
  const int t0 = c * kRwChunk, t1 = min(T, t0 + kRwChunk);
  for (int i = threadIdx.x; i < (t1 - t0) * E; i += kRwCols) sdl[i] = dlogits[static_cast<long long>(t0) * E + i];
  __syncthreads();
  if (h >= H) return;
  float acc[kMaxE];
#pragma unroll
  for (int e = 0; e < kMaxE; ++e) acc[e] = 0.f;
  for (int t = t0; t < t1; ++t) {
    const float xv = __bfloat162float(x[static_cast<long long>(t) * H + h]);
    const float* d = sdl + (t - t0) * E;
#pragma unroll
    for (int e = 0; e < kMaxE; ++e)
      if (e < E) acc[e] = fmaf(d[e], xv, acc[e]);
  }
#pragma unroll
  for (int e = 0; e < kMaxE; ++e)
    if (e < E) partial[(static_cast<long long>(c) * E + e) * H + h] = acc[e];
}

__global__ void moe_router_wgrad_reduce_kernel(const float* __restrict__ partial, int chunks, int E, int H,
                                               float* __restrict__ grad) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(E) * H) return;
  float s = 0.f;
  for (int c = 0; c < chunks; ++c) s += partial[static_cast<long long>(c) * E * H + i];
  grad[i] += s;
}

MoeRoutes make_routes(int world, int me, int E, int k, void* const* peers) {
  MoeRoutes r{};
  r.world = world;
  r.me = me;
  r.E = E;
  r.k = k;
  for (int i = 0; i < world; ++i) r.peers[i] = peers[i];
  return r;
}

}  // namespace

int moe_route(const void* x, const void* w, const float* bias, int T, int H, int E, int k, float* logits, int* topi,
              float* gates, cudaStream_t s) {
  if (E > kMaxE || k > kMaxK || k > E || H % 256) return -1;
  moe_route_kernel<<<(T * 32 + 255) / 256, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x),
                                                      reinterpret_cast<const __nv_bfloat16*>(w), bias, T, H, E, k,
                                                      logits, topi, gates);
  return static_cast<int>(cudaGetLastError());
}

int moe_positions(const int* topi, int n, int E, int* pos, int* counts, cudaStream_t s) {
  if (E > kMaxE) return -1;
  moe_positions_kernel<<<1, kPosThreads, 0, s>>>(topi, n, E, pos, counts);
  return static_cast<int>(cudaGetLastError());
}

int moe_dispatch(const void* x, const int* topi, const int* pos, int T, int k, int H, int world, int me, int E,
                 const int* period, const int* cycle, const int* cycle_rank, const int* per_cycle,
                 const long long* rowbase, void* const* recv, long long* route_row, cudaStream_t s) {
  if (world > kMaxE || E > kMaxE || H % 8) return -1;
  MoeRoutes r = make_routes(world, me, E, k, recv);
  r.period = period;
  r.cycle = cycle;
  r.cycle_rank = cycle_rank;
  r.per_cycle = per_cycle;
  r.rowbase = rowbase;
  const int n = T * k;
  moe_dispatch_kernel<<<(n * 32 + 255) / 256, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), topi, pos, n,
                                                         k, H, r, route_row);
  return static_cast<int>(cudaGetLastError());
}

int moe_combine(const void* residual, const float* gates, const long long* route_row, int T, int k, int H, int world,
                void* const* ybuf, void* out, void* ycache, cudaStream_t s) {
  if (world > kMaxE || H % 8) return -1;
  const MoeRoutes r = make_routes(world, 0, 0, k, ybuf);
  moe_combine_kernel<<<(T * 32 + 255) / 256, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(residual), gates,
                                                        route_row, T, k, H, r, reinterpret_cast<__nv_bfloat16*>(out),
                                                        reinterpret_cast<__nv_bfloat16*>(ycache));
  return static_cast<int>(cudaGetLastError());
}

int moe_grad_push(const void* dout, const float* gates, const void* ycache, const long long* route_row, int T, int k,
                  int H, int world, void* const* dyrecv, float* dgate, cudaStream_t s) {
  if (world > kMaxE || H % 8) return -1;
  const MoeRoutes r = make_routes(world, 0, 0, k, dyrecv);
  const int n = T * k;
  moe_grad_push_kernel<<<(n * 32 + 255) / 256, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(dout), gates,
                                                          reinterpret_cast<const __nv_bfloat16*>(ycache), route_row,
                                                          n, k, H, r, dgate);
  return static_cast<int>(cudaGetLastError());
}

int moe_grad_pull(const void* dout, const float* gates, const float* dgate, const int* topi,
                  const long long* route_row, int T, int k, int H, int E, int world, void* const* dxbuf, void* dx,
                  float* dlogits, cudaStream_t s, const void* router_w) {
  if (world > kMaxE || E > kMaxE || k > kMaxK || H % 8) return -1;
  const MoeRoutes r = make_routes(world, 0, E, k, dxbuf);
  moe_grad_pull_kernel<<<(T * 32 + 255) / 256, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(dout), gates,
                                                          dgate, topi, route_row, T, k, H, E, r,
                                                          reinterpret_cast<const __nv_bfloat16*>(router_w),
                                                          reinterpret_cast<__nv_bfloat16*>(dx), dlogits);
  return static_cast<int>(cudaGetLastError());
}

long long moe_router_wgrad_ws_floats(int T, int H, int E) {
  return static_cast<long long>((T + kRwChunk - 1) / kRwChunk) * E * H;
}

int moe_router_wgrad(const float* dlogits, const void* x, int T, int H, int E, float* partial, float* grad,
                     cudaStream_t s) {
  if (E > kMaxE || E <= 0 || T <= 0 || H <= 0) return -1;
  const int chunks = (T + kRwChunk - 1) / kRwChunk;
  moe_router_wgrad_kernel<<<dim3((H + kRwCols - 1) / kRwCols, chunks), kRwCols, 0, s>>>(
      dlogits, reinterpret_cast<const __nv_bfloat16*>(x), T, H, E, partial);
  const long long n = static_cast<long long>(E) * H;
  moe_router_wgrad_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(partial, chunks, E, H, grad);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rb
