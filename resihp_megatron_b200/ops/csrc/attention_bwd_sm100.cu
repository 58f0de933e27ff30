// Causal GQA flash-attention backward on tcgen05 tensor cores (head dim 128), deterministic.
//
// Two kernels after a small prep kernel (delta = rowsum(dO * O), nl2 = -lse * log2(e)):
//
//   dK/dV: one CTA per (key block j of 128 keys, kv head, batch), looping over the q heads of
//   the group and the query blocks i >= j.  The transposed problem keeps one key per TMEM lane:
//     S^T  = K_j Q_i^T       (SS MMA, both K-major)           TMEM cols [  0,128)
//     dP^T = V_j dO_i^T      (SS MMA, both K-major)           TMEM cols [128,256)
//     P^T  = exp2(S^T * scale*log2e + nl2[q]),  dS^T = P^T * (dP^T - delta[q])
//     dV  += P^T dO_i        (TS MMA: A = P^T from TMEM, B = dO MN-major) cols [256,384)
//     dK  += dS^T Q_i        (TS MMA: A = dS^T from TMEM, B = Q MN-major) cols [384,512)
//   P^T and dS^T are written back (bf16 pairs) over the first half of the columns they came
//   from, so no shared memory is spent on them; Q_i / dO_i / nl2 / delta stream through a
//   2-stage TMA ring.  The issue order dV(i), S(i+1), dK(i), dP(i+1) lets the tensor core run
//   while the softmax warps work: tcgen05 MMAs of one thread execute in issue order, so S(i+1)
//   overwrites P^T(i) only after dV(i) consumed it.
//
//   dQ: one CTA per (query block i, q head, batch), looping over key blocks j <= i with one
//   query per TMEM lane: S = Q_i K_j^T, dP = dO_i V_j^T, dS = P * (dP - delta), dQ += dS K_j
//   (TS MMA).  S(j+1) is issued as soon as the softmax warps have read S(j).
//
// dQ is recomputed in its own kernel instead of accumulated with atomics, so every gradient is
// a fixed-order sum: bit-identical run to run.  Roles (320 threads): warps 0-7 softmax (warp w
// owns TMEM lanes 32*(w%4).. and column half w/4), warp 8 TMA producer, warp 9 TMEM allocator
// and MMA issuer.  Every mbarrier wait is bounded; a timeout unwinds all roles, sets the error
// word and the kernel returns.  No TMA multicast is used.
//
// The reference (Megatron-Core + TransformerEngine attention) has no kernel of its own here; this
// is the backward of the forward in attention_sm100.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include <cstdint>

#include "kernels.h"
#include "exp2_fma.cuh"
#include "sm100.cuh"

namespace rb {

int make_tmap_bf16_2d(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                      uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int kTile = 128;
constexpr int kTileBytes = kTile * kTile * 2;  // 32 KB: two 128B-swizzled halves of 64 columns
constexpr int kHalf = kTileBytes / 2;
constexpr int kThreads = 320;
constexpr int kVecBytes = kTile * 4;  // one block of nl2 or delta
constexpr int kSmemDkdv = 1024 + 6 * kTileBytes + 4 * kVecBytes + 256;
constexpr int kSmemDq = 1024 + 6 * kTileBytes + 256;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  const float* nl2;    // -lse * log2(e), [B, Hq, S]
  const float* delta;  // [B, Hq, S]
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  long long dq_stride, dk_stride, dv_stride;
  int B, S, Hq, Hkv;
  float scale, scale_log2;
  int* err;
};

__device__ __forceinline__ bool warp_wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int s) {
  return make_smem_desc(base + (s >> 2) * kHalf + (s & 3) * 32, 16, 1024, kSwizzle128B);
}

__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int s) {
  return make_smem_desc(base + s * 2048, kHalf, 1024, kSwizzle128B);
}

// TMEM column of the packed bf16 A operand for k-step s: k-steps 0-3 live in the first 32
// columns of the region, 4-7 at +64 (each column half is written by its own warp group).
__device__ __forceinline__ uint32_t packed_col(int s) { return (s >> 2) * 64 + (s & 3) * 8; }

// Load 64 fp32 columns of this thread's TMEM lane.
// Both 32-column loads are in flight before the one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t addr, float (&v)[64]) {
  uint32_t t[2][32];
  tmem_ld_32x32b_x32(addr, t[0]);
  tmem_ld_32x32b_x32(addr + 32, t[1]);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(t[i >> 5][i & 31]);
}

// Write 64 fp32 values of this thread's row as bf16 to global memory (128 contiguous bytes).
__device__ __forceinline__ void store_row64(__nv_bfloat16* dst, uint32_t taddr, float mul) {
  uint32_t t[32];
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    tmem_ld_32x32b_x32(taddr + c * 32, t);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 u;
      u.x = pack_bf16x2(__uint_as_float(t[8 * i + 0]) * mul, __uint_as_float(t[8 * i + 1]) * mul);
      u.y = pack_bf16x2(__uint_as_float(t[8 * i + 2]) * mul, __uint_as_float(t[8 * i + 3]) * mul);
      u.z = pack_bf16x2(__uint_as_float(t[8 * i + 4]) * mul, __uint_as_float(t[8 * i + 5]) * mul);
      u.w = pack_bf16x2(__uint_as_float(t[8 * i + 6]) * mul, __uint_as_float(t[8 * i + 7]) * mul);
      *reinterpret_cast<uint4*>(dst + c * 32 + 8 * i) = u;
    }
  }
}

// ------------------------------------------------------------------------------ prep
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, long long o_stride,
                                     const __nv_bfloat16* __restrict__ dout, long long do_stride,
                                     const float* __restrict__ lse, float* __restrict__ delta,
                                     float* __restrict__ nl2, int B, int S, int Hq) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(B) * S * Hq) return;
  const int h = static_cast<int>(w % Hq);
  const long long row = w / Hq;
  const int b = static_cast<int>(row / S), s = static_cast<int>(row % S);
  const uint2 ov = *reinterpret_cast<const uint2*>(o + row * o_stride + h * kTile + lane * 4);
  const uint2 dv = *reinterpret_cast<const uint2*>(dout + row * do_stride + h * kTile + lane * 4);
  const float2 o0 = unpack_bf16x2(ov.x), o1 = unpack_bf16x2(ov.y);
  const float2 d0 = unpack_bf16x2(dv.x), d1 = unpack_bf16x2(dv.y);
  float acc = o0.x * d0.x + o0.y * d0.y + o1.x * d1.x + o1.y * d1.y;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const long long idx = (static_cast<long long>(b) * Hq + h) * S + s;
    delta[idx] = acc;
    nl2[idx] = -lse[idx] * kLog2e;
  }
}

// ------------------------------------------------------------------------------ dK / dV
template <int kFma>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dkdv_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                               BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTileBytes;
  uint8_t* sQ = smem + 2 * kTileBytes;   // 2 stages
  uint8_t* sdO = smem + 4 * kTileBytes;  // 2 stages
  float* sL = reinterpret_cast<float*>(smem + 6 * kTileBytes);  // 2 stages of nl2
  float* sD = sL + 2 * kTile;                                     // 2 stages of delta
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kTileBytes + 4 * kVecBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar_kv = smem_u32(&bars[0]);
  auto bar_qf = [&](int st) { return smem_u32(&bars[1 + st]); };
  auto bar_qe = [&](int st) { return smem_u32(&bars[3 + st]); };
  const uint32_t bar_s = smem_u32(&bars[5]), bar_dp = smem_u32(&bars[6]);
  const uint32_t bar_p = smem_u32(&bars[7]), bar_ds = smem_u32(&bars[8]);
  const uint32_t bar_acc = smem_u32(&bars[9]), bar_final = smem_u32(&bars[10]);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = p.S / kTile;
  // heaviest tasks (smallest key block) first
  const int per_j = p.Hkv * p.B;
  const int j = blockIdx.x / per_j;
  const int hk = (blockIdx.x % per_j) % p.Hkv;
  const int b = (blockIdx.x % per_j) / p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int per_head = nkb - j;
  const int n_it = group * per_head;
  const int row_base = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar_qf(st), 1);
      mbar_init(bar_qe(st), 1);
    }
    mbar_init(bar_s, 1);
    mbar_init(bar_dp, 1);
    mbar_init(bar_p, 8);
    mbar_init(bar_ds, 8);
    mbar_init(bar_acc, 1);
    mbar_init(bar_final, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(bar_kv, 2 * kTileBytes);
      for (int hf = 0; hf < 2; ++hf) {
        tma_load_2d(smem_u32(sK + hf * kHalf), &tmK, bar_kv, hk * kTile + hf * 64, row_base + j * kTile);
        tma_load_2d(smem_u32(sV + hf * kHalf), &tmV, bar_kv, hk * kTile + hf * 64, row_base + j * kTile);
      }
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int st = it & 1;
        if (!mbar_wait(bar_qe(st), ((it >> 1) & 1) ^ 1, abort_flag, p.err)) break;
        const int hh = hk * group + it / per_head;
        const int i = j + it % per_head;
        mbar_arrive_expect_tx(bar_qf(st), 2 * kTileBytes + 2 * kVecBytes);
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_2d(smem_u32(sQ + st * kTileBytes + hf * kHalf), &tmQ, bar_qf(st), hh * kTile + hf * 64,
                      row_base + i * kTile);
          tma_load_2d(smem_u32(sdO + st * kTileBytes + hf * kHalf), &tmdO, bar_qf(st), hh * kTile + hf * 64,
                      row_base + i * kTile);
        }
        const long long vec = (static_cast<long long>(b) * p.Hq + hh) * p.S + i * kTile;
        bulk_load_1d(smem_u32(sL + st * kTile), p.nl2 + vec, kVecBytes, bar_qf(st));
        bulk_load_1d(smem_u32(sD + st * kTile), p.delta + vec, kVecBytes, bar_qf(st));
        issued = it + 1;
      }
      // drain: every load issued must land before the CTA may exit
      mbar_wait(bar_kv, 0, nullptr, p.err, 200000000ull);
      for (int it = issued > 2 ? issued - 2 : 0; it < issued; ++it)
        mbar_wait(bar_qf(it & 1), (it >> 1) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_ss = make_idesc_f16(128, 128, true, false, false);
      constexpr uint32_t idesc_ts = make_idesc_f16(128, 128, true, false, true);
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sdO);
      bool ok = mbar_wait(bar_kv, 0, abort_flag, p.err);
      auto issue_s = [&](int it) {
        const int st = it & 1;
        if (!mbar_wait(bar_qf(st), (it >> 1) & 1, abort_flag, p.err)) return false;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16(tS, kmajor_desc(k_base, s), kmajor_desc(q_base + st * kTileBytes, s), idesc_ss, s > 0);
        umma_commit(bar_s);
        return true;
      };
      auto issue_dp = [&](int it) {
        const int st = it & 1;
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16(tdP, kmajor_desc(v_base, s), kmajor_desc(do_base + st * kTileBytes, s), idesc_ss, s > 0);
        umma_commit(bar_dp);
      };
      if (ok && (ok = issue_s(0))) issue_dp(0);
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it & 1;
        if (!(ok = mbar_wait(bar_p, it & 1, abort_flag, p.err))) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16_ts(tdV, tS + packed_col(s), mnmajor_desc(do_base + st * kTileBytes, s), idesc_ts,
                      (it > 0 || s > 0) ? 1u : 0u);
        if (it + 1 < n_it && !(ok = issue_s(it + 1))) break;
        if (!(ok = mbar_wait(bar_ds, it & 1, abort_flag, p.err))) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16_ts(tdK, tdP + packed_col(s), mnmajor_desc(q_base + st * kTileBytes, s), idesc_ts,
                      (it > 0 || s > 0) ? 1u : 0u);
        umma_commit(bar_qe(st));
        if (it + 1 < n_it) issue_dp(it + 1);
      }
      if (ok) umma_commit(bar_acc);
      // every MMA this thread issued completes before TMEM is released
      umma_commit(bar_final);
      mbar_wait(bar_final, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int X = warp >> 2;                // column half (queries X*64 .. X*64+63)
    const int r = (warp & 3) * 32 + lane;   // key row in the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int st = it & 1;
      const int i = j + it % per_head;
      if (!(ok = warp_wait_bar(bar_qf(st), (it >> 1) & 1, abort_flag, p.err))) break;
      if (!(ok = warp_wait_bar(bar_s, it & 1, abort_flag, p.err))) break;
      tc_fence_after();
      float pv[64];
      tmem_ld64(tS + lane_off + X * 64, pv);
      const float* nl = sL + st * kTile + X * 64;
      const bool diag = i == j;
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 l4 = *reinterpret_cast<const float4*>(nl + c4 * 4);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = c4 * 4 + e;
          float x = ex2_mixed<kFma>(fmaf(pv[c], p.scale_log2, lv[e]), c);
          if (diag && X * 64 + c < r) x = 0.f;  // query before key: masked
          pv[c] = x;
        }
      }
      {
        uint32_t t[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) t[c] = pack_bf16x2(pv[2 * c], pv[2 * c + 1]);
        tmem_st_32x32b_x32(tS + lane_off + X * 64, t);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p);
      if (!(ok = warp_wait_bar(bar_dp, it & 1, abort_flag, p.err))) break;
      tc_fence_after();
      const float* dl = sD + st * kTile + X * 64;
      {
        uint32_t t[32], out[32];
#pragma unroll
        for (int c32 = 0; c32 < 2; ++c32) {
          tmem_ld_32x32b_x32(tdP + lane_off + X * 64 + c32 * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            const float4 d4 = *reinterpret_cast<const float4*>(dl + c32 * 32 + c4 * 4);
            const int c = c32 * 32 + c4 * 4;
            const float a0 = pv[c + 0] * (__uint_as_float(t[c4 * 4 + 0]) - d4.x);
            const float a1 = pv[c + 1] * (__uint_as_float(t[c4 * 4 + 1]) - d4.y);
            const float a2 = pv[c + 2] * (__uint_as_float(t[c4 * 4 + 2]) - d4.z);
            const float a3 = pv[c + 3] * (__uint_as_float(t[c4 * 4 + 3]) - d4.w);
            out[c32 * 16 + c4 * 2 + 0] = pack_bf16x2(a0, a1);
            out[c32 * 16 + c4 * 2 + 1] = pack_bf16x2(a2, a3);
          }
        }
        tmem_st_32x32b_x32(tdP + lane_off + X * 64, out);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_ds);
    }
    if (ok && warp_wait_bar(bar_acc, 0, abort_flag, p.err)) {
      tc_fence_after();
      const long long key = row_base + j * kTile + r;
      store_row64(p.dv + key * p.dv_stride + hk * kTile + X * 64, tdV + lane_off + X * 64, 1.f);
      store_row64(p.dk + key * p.dk_stride + hk * kTile + X * 64, tdK + lane_off + X * 64, p.scale);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------ dQ
template <int kFma>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dq_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                             BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = smem + kTileBytes;
  uint8_t* sK = smem + 2 * kTileBytes;  // 2 stages
  uint8_t* sV = smem + 4 * kTileBytes;  // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar_q = smem_u32(&bars[0]);
  auto bar_kvf = [&](int st) { return smem_u32(&bars[1 + st]); };
  auto bar_kve = [&](int st) { return smem_u32(&bars[3 + st]); };
  const uint32_t bar_s = smem_u32(&bars[5]), bar_sfree = smem_u32(&bars[6]);
  const uint32_t bar_dp = smem_u32(&bars[7]), bar_ds = smem_u32(&bars[8]);
  const uint32_t bar_acc = smem_u32(&bars[9]), bar_final = smem_u32(&bars[10]);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.S / kTile;
  const int per_i = p.Hq * p.B;
  const int i = nqb - 1 - static_cast<int>(blockIdx.x / per_i);  // heaviest (latest) query blocks first
  const int h = (blockIdx.x % per_i) % p.Hq;
  const int b = (blockIdx.x % per_i) / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int n_it = i + 1;
  const int row_base = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar_kvf(st), 1);
      mbar_init(bar_kve(st), 1);
    }
    mbar_init(bar_s, 1);
    mbar_init(bar_sfree, 8);
    mbar_init(bar_dp, 1);
    mbar_init(bar_ds, 8);
    mbar_init(bar_acc, 1);
    mbar_init(bar_final, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdQ = tmem + 256;

  if (warp == 8) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(bar_q, 2 * kTileBytes);
      for (int hf = 0; hf < 2; ++hf) {
        tma_load_2d(smem_u32(sQ + hf * kHalf), &tmQ, bar_q, h * kTile + hf * 64, row_base + i * kTile);
        tma_load_2d(smem_u32(sdO + hf * kHalf), &tmdO, bar_q, h * kTile + hf * 64, row_base + i * kTile);
      }
      int issued = 0;
      for (int jj = 0; jj < n_it; ++jj) {
        const int st = jj & 1;
        if (!mbar_wait(bar_kve(st), ((jj >> 1) & 1) ^ 1, abort_flag, p.err)) break;
        mbar_arrive_expect_tx(bar_kvf(st), 2 * kTileBytes);
        for (int hf = 0; hf < 2; ++hf) {
          tma_load_2d(smem_u32(sK + st * kTileBytes + hf * kHalf), &tmK, bar_kvf(st), hk * kTile + hf * 64,
                      row_base + jj * kTile);
          tma_load_2d(smem_u32(sV + st * kTileBytes + hf * kHalf), &tmV, bar_kvf(st), hk * kTile + hf * 64,
                      row_base + jj * kTile);
        }
        issued = jj + 1;
      }
      mbar_wait(bar_q, 0, nullptr, p.err, 200000000ull);
      for (int jj = issued > 2 ? issued - 2 : 0; jj < issued; ++jj)
        mbar_wait(bar_kvf(jj & 1), (jj >> 1) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc_ss = make_idesc_f16(128, 128, true, false, false);
      constexpr uint32_t idesc_ts = make_idesc_f16(128, 128, true, false, true);
      const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sdO);
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      bool ok = mbar_wait(bar_q, 0, abort_flag, p.err);
      auto issue_s = [&](int jj) {
        const int st = jj & 1;
        if (!mbar_wait(bar_kvf(st), (jj >> 1) & 1, abort_flag, p.err)) return false;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16(tS, kmajor_desc(q_base, s), kmajor_desc(k_base + st * kTileBytes, s), idesc_ss, s > 0);
        umma_commit(bar_s);
        return true;
      };
      auto issue_dp = [&](int jj) {
        const int st = jj & 1;
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16(tdP, kmajor_desc(do_base, s), kmajor_desc(v_base + st * kTileBytes, s), idesc_ss, s > 0);
        umma_commit(bar_dp);
      };
      if (ok && (ok = issue_s(0))) issue_dp(0);
      for (int jj = 0; ok && jj < n_it; ++jj) {
        const int st = jj & 1;
        if (jj + 1 < n_it) {
          if (!(ok = mbar_wait(bar_sfree, jj & 1, abort_flag, p.err))) break;
          tc_fence_after();
          if (!(ok = issue_s(jj + 1))) break;
        }
        if (!(ok = mbar_wait(bar_ds, jj & 1, abort_flag, p.err))) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16_ts(tdQ, tdP + packed_col(s), mnmajor_desc(k_base + st * kTileBytes, s), idesc_ts,
                      (jj > 0 || s > 0) ? 1u : 0u);
        umma_commit(bar_kve(st));
        if (jj + 1 < n_it) issue_dp(jj + 1);
      }
      if (ok) umma_commit(bar_acc);
      umma_commit(bar_final);
      mbar_wait(bar_final, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    const int X = warp >> 2;               // column half (keys X*64 .. X*64+63)
    const int r = (warp & 3) * 32 + lane;  // query row in the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const long long vec = (static_cast<long long>(b) * p.Hq + h) * p.S + i * kTile + r;
    const float nl = p.nl2[vec];
    const float dl = p.delta[vec];
    bool ok = true;
    for (int jj = 0; jj < n_it; ++jj) {
      if (!(ok = warp_wait_bar(bar_s, jj & 1, abort_flag, p.err))) break;
      tc_fence_after();
      float pv[64];
      tmem_ld64(tS + lane_off + X * 64, pv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree);
      const bool diag = jj == i;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        float x = ex2_mixed<kFma>(fmaf(pv[c], p.scale_log2, nl), c);
        if (diag && X * 64 + c > r) x = 0.f;  // key after query: masked
        pv[c] = x;
      }
      if (!(ok = warp_wait_bar(bar_dp, jj & 1, abort_flag, p.err))) break;
      tc_fence_after();
      {
        uint32_t t[2][32], out[32];
        tmem_ld_32x32b_x32(tdP + lane_off + X * 64, t[0]);
        tmem_ld_32x32b_x32(tdP + lane_off + X * 64 + 32, t[1]);
        tmem_ld_wait();
#pragma unroll
        for (int c32 = 0; c32 < 2; ++c32) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float a0 = pv[c32 * 32 + 2 * c] * (__uint_as_float(t[c32][2 * c]) - dl);
            const float a1 = pv[c32 * 32 + 2 * c + 1] * (__uint_as_float(t[c32][2 * c + 1]) - dl);
            out[c32 * 16 + c] = pack_bf16x2(a0, a1);
          }
        }
        tmem_st_32x32b_x32(tdP + lane_off + X * 64, out);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_ds);
    }
    if (ok && warp_wait_bar(bar_acc, 0, abort_flag, p.err)) {
      tc_fence_after();
      const long long q = row_base + i * kTile + r;
      store_row64(p.dq + q * p.dq_stride + h * kTile + X * 64, tdQ + lane_off + X * 64, p.scale);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool misaligned(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) != 0; }

// A second stream of the current device with its fork / join events, created on first use and
// kept for the life of the process; stream == nullptr if creation failed (then one stream is used).
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

SideStream& side_stream() {
  constexpr int kMaxDevices = 64;
  static SideStream per_device[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    static SideStream none;
    return none;
  }
  std::lock_guard<std::mutex> lock(mu);
  SideStream& s = per_device[dev];
  if (s.stream == nullptr) {
    cudaStream_t st = nullptr;
    cudaEvent_t f = nullptr, j = nullptr;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
        cudaEventCreateWithFlags(&f, cudaEventDisableTiming) == cudaSuccess &&
        cudaEventCreateWithFlags(&j, cudaEventDisableTiming) == cudaSuccess) {
      s.stream = st;
      s.fork = f;
      s.join = j;
    } else {
      cudaGetLastError();  // clear; the caller falls back to one stream
    }
  }
  return s;
}

// Exponentials per 8 score columns evaluated on the FMA pipe (ex2_fma) by default.  Measured on
// B200 at B=2 S=4096 (forward / backward TFLOP/s for shares 0..3): 797/585, 768/581, 751/572,
// 732/561 -- with the softmax's dependency chains broken up the MUFU unit is not the limit, so
// every exponential stays on MUFU; the other shares remain selectable for tuning.
constexpr int kDefaultFmaShare = 0;

template <int kFma>
int launch_bwd(dim3 grid_dkdv, dim3 grid_dq, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
               const CUtensorMap& tdo, const BwdParams& p, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_bwd_dkdv_sm100_kernel<kFma>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemDkdv);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_bwd_dq_sm100_kernel<kFma>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kSmemDq);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr = true;
  }
  // dK/dV and dQ read the same inputs and write disjoint outputs: dQ runs on a second stream so
  // its CTAs fill the SMs the dK/dV grid's partial last wave leaves idle (and the other way
  // round); the caller's stream waits for both.  Each output is still computed by one fixed CTA.
  SideStream& side = side_stream();
  if (side.stream == nullptr) {
    attn_bwd_dkdv_sm100_kernel<kFma><<<grid_dkdv, kThreads, kSmemDkdv, stream>>>(tq, tk, tv, tdo, p);
    attn_bwd_dq_sm100_kernel<kFma><<<grid_dq, kThreads, kSmemDq, stream>>>(tq, tk, tv, tdo, p);
    return static_cast<int>(cudaGetLastError());
  }
  cudaError_t e = cudaEventRecord(side.fork, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(side.stream, side.fork, 0);
  if (e != cudaSuccess) return static_cast<int>(e);
  attn_bwd_dkdv_sm100_kernel<kFma><<<grid_dkdv, kThreads, kSmemDkdv, stream>>>(tq, tk, tv, tdo, p);
  attn_bwd_dq_sm100_kernel<kFma><<<grid_dq, kThreads, kSmemDq, side.stream>>>(tq, tk, tv, tdo, p);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaEventRecord(side.join, side.stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, side.join, 0);
  return static_cast<int>(e);
}

}  // namespace

// Returns 1 when the shape is not handled here (the caller uses the mma.sync path).
// `nl2` is scratch of B * Hq * S floats; `a.delta` receives rowsum(dO * O).  ``variant``:
// exponentials per 8 score columns on the FMA pipe (0-3), or -1 for the default.
int attention_bwd_sm100(const AttnBwdArgs& a, int D, float* nl2, int* err, cudaStream_t stream, int variant) {
  if (D != 128 || !a.causal || a.S % kTile != 0 || a.Hq % a.Hkv != 0) return 1;
  if (misaligned(a.q) || misaligned(a.k) || misaligned(a.v) || misaligned(a.o) || misaligned(a.dout) ||
      misaligned(a.dq) || misaligned(a.dk) || misaligned(a.dv) || misaligned(a.lse) || misaligned(a.delta) ||
      misaligned(nl2))
    return 1;
  if ((a.q_stride | a.k_stride | a.v_stride | a.o_stride | a.do_stride | a.dq_stride | a.dk_stride | a.dv_stride) & 7)
    return 1;
  const long long T = static_cast<long long>(a.B) * a.S;
  {
    const long long warps = T * a.Hq;
    const int blocks = static_cast<int>((warps * 32 + 255) / 256);
    attn_bwd_prep_kernel<<<blocks, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(a.o), a.o_stride, reinterpret_cast<const __nv_bfloat16*>(a.dout),
        a.do_stride, a.lse, a.delta, nl2, a.B, a.S, a.Hq);
  }
  CUtensorMap tq, tk, tv, tdo;
  if (make_tmap_bf16_2d(&tq, a.q, static_cast<uint64_t>(a.Hq) * kTile, T, a.q_stride, 64, kTile)) return -20;
  if (make_tmap_bf16_2d(&tk, a.k, static_cast<uint64_t>(a.Hkv) * kTile, T, a.k_stride, 64, kTile)) return -21;
  if (make_tmap_bf16_2d(&tv, a.v, static_cast<uint64_t>(a.Hkv) * kTile, T, a.v_stride, 64, kTile)) return -22;
  if (make_tmap_bf16_2d(&tdo, a.dout, static_cast<uint64_t>(a.Hq) * kTile, T, a.do_stride, 64, kTile)) return -23;
  BwdParams p{nl2,
              a.delta,
              reinterpret_cast<__nv_bfloat16*>(a.dq),
              reinterpret_cast<__nv_bfloat16*>(a.dk),
              reinterpret_cast<__nv_bfloat16*>(a.dv),
              a.dq_stride,
              a.dk_stride,
              a.dv_stride,
              a.B,
              a.S,
              a.Hq,
              a.Hkv,
              a.scale,
              a.scale * kLog2e,
              err};
  const int nb = a.S / kTile;
  const dim3 grid_dkdv(nb * a.Hkv * a.B), grid_dq(nb * a.Hq * a.B);
  switch (variant < 0 ? kDefaultFmaShare : variant) {
    case 0: return launch_bwd<0>(grid_dkdv, grid_dq, tq, tk, tv, tdo, p, stream);
    case 1: return launch_bwd<1>(grid_dkdv, grid_dq, tq, tk, tv, tdo, p, stream);
    case 2: return launch_bwd<2>(grid_dkdv, grid_dq, tq, tk, tv, tdo, p, stream);
    case 3: return launch_bwd<3>(grid_dkdv, grid_dq, tq, tk, tv, tdo, p, stream);
    default: return -24;
  }
}

}  // namespace rb
