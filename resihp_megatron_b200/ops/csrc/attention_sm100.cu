// Causal GQA flash-attention forward on tcgen05 tensor cores (head dim 128).
//
// CTA = 256 query rows of one (batch, head): two 128-row tiles A and B that share every K/V
// block.  Roles (320 threads):
//   warps 0-3  softmax + epilogue of tile A (thread = query row = TMEM lane)
//   warps 4-7  softmax + epilogue of tile B
//   warp 8     TMA producer: Q_A, Q_B once, then K_j and V_j (128 x 128 bf16 each)
//   warp 9     TMEM allocator and single-thread MMA issuer
// TMEM (512 columns): S_A | S_B | O_A | O_B, 128 fp32 columns each.
// Per key block j:  S_X = Q_X K_j^T (tcgen05, both operands K-major from shared memory);
// softmax reads its S row from TMEM, applies the causal mask on the diagonal block, updates the
// running max, and writes P (bf16 pairs) back over the first half of S_X's TMEM columns; then
// O_X += P_X V_j with P read from TMEM (TS MMA) and V as an MN-major operand.  K and V are
// double-buffered.  The MMA issue order PV_A(j), S_A(j+1), PV_B(j), S_B(j+1) lets one tile's
// softmax overlap the other tile's MMAs.  O stays in TMEM; it is rescaled (TMEM load / multiply
// / store) only when a row's max grows by more than 2^8, so the common case costs nothing -- l
// and O always share the same reference max, so the result is exact.  Output rows are
// normalised by l in the epilogue and LSE is written for the backward.
//
// Every mbarrier wait is bounded (see sm100.cuh); a timeout unwinds all roles and the kernel
// returns with an error word set.  No TMA multicast is used.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "exp2_fma.cuh"
#include "sm100.cuh"

namespace rb {

int make_tmap_bf16_2d(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                      uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int kTile = 128;                    // rows of a Q tile / K block, and the head dim
constexpr int kTileBytes = kTile * kTile * 2;  // 32 KB: two 16 KB halves of 64 columns
constexpr int kHalf = kTileBytes / 2;
constexpr int kThreads = 320;
constexpr int kSmem = 1024 + 6 * kTileBytes + 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdParams {
  __nv_bfloat16* o;
  long long o_stride;
  float* lse;
  int B, S, Hq, Hkv;
  float scale_log2;  // softmax scale * log2(e)
  int* err;
};

__device__ __forceinline__ bool warp_wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ float ex2(float x) { return ex2_mufu(x); }

// K-major operand descriptor for k-step s (16 columns) of a [128 x 128] tile stored as two
// 128B-swizzled halves of 64 columns.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int s) {
  return make_smem_desc(base + (s >> 2) * kHalf + (s & 3) * 32, 16, 1024, kSwizzle128B);
}

// MN-major operand descriptor (V: N = head dim in two 64-wide halves, K = key rows) for k-step s.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int s) {
  return make_smem_desc(base + s * 2048, kHalf, 1024, kSwizzle128B);
}

template <int kFma>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // Q_A, Q_B
  uint8_t* sK = smem + 2 * kTileBytes;  // 2 stages
  uint8_t* sV = smem + 4 * kTileBytes;  // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar_q = smem_u32(&bars[0]);
  auto bar_kf = [&](int st) { return smem_u32(&bars[1 + st]); };
  auto bar_ke = [&](int st) { return smem_u32(&bars[3 + st]); };
  auto bar_vf = [&](int st) { return smem_u32(&bars[5 + st]); };
  auto bar_ve = [&](int st) { return smem_u32(&bars[7 + st]); };
  auto bar_s = [&](int x) { return smem_u32(&bars[9 + x]); };
  auto bar_p = [&](int x) { return smem_u32(&bars[11 + x]); };
  auto bar_o = [&](int x) { return smem_u32(&bars[13 + x]); };
  const uint32_t bar_final = smem_u32(&bars[15]);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heaviest (latest) query blocks first across the whole grid
  const int per_qb = p.Hq * p.B;
  const int nqb = p.S / (2 * kTile);
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x / per_qb);
  const int h = (blockIdx.x % per_qb) % p.Hq;
  const int b = (blockIdx.x % per_qb) / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qb * 2 * kTile;
  const int jA = 2 * qb, jB = 2 * qb + 1;  // last key block of tile A / tile B
  const int nkv = jB + 1;
  const int row_base = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar_kf(st), 1);
      mbar_init(bar_ke(st), 1);
      mbar_init(bar_vf(st), 1);
      mbar_init(bar_ve(st), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bar_s(x), 1);
      mbar_init(bar_p(x), 4);
      mbar_init(bar_o(x), 1);
    }
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
  const uint32_t tmem = *tmem_slot;  // columns: S_A | S_B | O_A | O_B

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(bar_q, 2 * kTileBytes);
      for (int x = 0; x < 2; ++x)
        for (int hf = 0; hf < 2; ++hf)
          tma_load_2d(smem_u32(sQ + x * kTileBytes + hf * kHalf), &tmQ, bar_q, h * kTile + hf * 64,
                      row_base + q0 + x * kTile);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(bar_ke(st), ((j >> 1) & 1) ^ 1, abort_flag, p.err)) break;
        mbar_arrive_expect_tx(bar_kf(st), kTileBytes);
        for (int hf = 0; hf < 2; ++hf)
          tma_load_2d(smem_u32(sK + st * kTileBytes + hf * kHalf), &tmK, bar_kf(st), hk * kTile + hf * 64,
                      row_base + j * kTile);
        issued_k = j + 1;
        if (!mbar_wait(bar_ve(st), ((j >> 1) & 1) ^ 1, abort_flag, p.err)) break;
        mbar_arrive_expect_tx(bar_vf(st), kTileBytes);
        for (int hf = 0; hf < 2; ++hf)
          tma_load_2d(smem_u32(sV + st * kTileBytes + hf * kHalf), &tmV, bar_vf(st), hk * kTile + hf * 64,
                      row_base + j * kTile);
        issued_v = j + 1;
      }
      // drain: the last loads issued must land before the CTA may exit
      mbar_wait(bar_q, 0, nullptr, p.err, 200000000ull);
      for (int j = issued_k > 2 ? issued_k - 2 : 0; j < issued_k; ++j)
        mbar_wait(bar_kf(j & 1), (j >> 1) & 1, nullptr, p.err, 200000000ull);
      for (int j = issued_v > 2 ? issued_v - 2 : 0; j < issued_v; ++j)
        mbar_wait(bar_vf(j & 1), (j >> 1) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    // Order per key block j: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1).  While the softmax warps of one
    // tile work on their S, the tensor cores run the other tile's two MMAs.  tcgen05 MMAs of one
    // thread execute in issue order, so S_X(j+1) overwrites P_X(j) (kept in S_X's columns) only
    // after PV_X(j) consumed it.
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(128, 128, true, false, false);
      constexpr uint32_t idesc_o = make_idesc_f16(128, 128, true, false, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto issue_s = [&](int x, int j) {
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16(tmem + x * 128, kmajor_desc(q_base + x * kTileBytes, s),
                   kmajor_desc(k_base + (j & 1) * kTileBytes, s), idesc_s, s > 0 ? 1u : 0u);
        umma_commit(bar_s(x));
      };
      auto issue_pv = [&](int x, int j) {
#pragma unroll
        for (int s = 0; s < 8; ++s)
          umma_f16_ts(tmem + 256 + x * 128, tmem + x * 128 + s * 8, mnmajor_desc(v_base + (j & 1) * kTileBytes, s),
                      idesc_o, (j > 0 || s > 0) ? 1u : 0u);
        umma_commit(bar_o(x));
      };
      bool ok = mbar_wait(bar_q, 0, abort_flag, p.err) && mbar_wait(bar_kf(0), 0, abort_flag, p.err);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(bar_ke(0));
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j & 1;
        const int nx = j + 1;
        if (!(ok = mbar_wait(bar_vf(st), (j >> 1) & 1, abort_flag, p.err))) break;
        bool k_waited = false;
        if (j <= jA) {
          if (!(ok = mbar_wait(bar_p(0), j & 1, abort_flag, p.err))) break;
          tc_fence_after();
          issue_pv(0, j);
          if (nx <= jA) {
            if (!(ok = mbar_wait(bar_kf(nx & 1), (nx >> 1) & 1, abort_flag, p.err))) break;
            k_waited = true;
            tc_fence_after();
            issue_s(0, nx);
          }
        }
        if (!(ok = mbar_wait(bar_p(1), j & 1, abort_flag, p.err))) break;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(bar_ve(st));
        if (nx <= jB) {
          if (!k_waited) {
            if (!(ok = mbar_wait(bar_kf(nx & 1), (nx >> 1) & 1, abort_flag, p.err))) break;
            tc_fence_after();
          }
          issue_s(1, nx);
          umma_commit(bar_ke(nx & 1));
        }
      }
      // every MMA this thread issued completes before TMEM is released
      umma_commit(bar_final);
      mbar_wait(bar_final, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int X = warp >> 2;                 // tile
    const int r = (warp & 3) * 32 + lane;    // row in tile == TMEM lane
    const int jmax = X == 0 ? jA : jB;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + X * 128;
    const uint32_t o_addr = tmem + lane_off + 256 + X * 128;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j <= jmax; ++j) {
      if (!(ok = warp_wait_bar(bar_s(X), j & 1, abort_flag, p.err))) break;
      tc_fence_after();
      // Two passes over S in 64-column halves (two 32-column loads in flight per wait): the row max
      // first, then P.  Re-reading S from TMEM is cheap and keeps 64 scores, not 128, in registers.
      // The diagonal block masks key > query to -inf.
      const bool diag = j == jmax;
      float m8[8];  // 8 independent max chains: one chain of dependent max operations is latency bound
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t t[2][32];
        tmem_ld_32x32b_x32(s_addr + half * 64, t[0]);
        tmem_ld_32x32b_x32(s_addr + half * 64 + 32, t[1]);
        tmem_ld_wait();
        if (diag) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (half * 64 + c > r) t[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 0; c < 64; ++c) m8[c & 7] = fmaxf(m8[c & 7], __uint_as_float(t[c >> 5][c & 31]));
      }
      // the scale is positive, so the max of scaled scores is the scaled raw max
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * p.scale_log2;
      const bool need = mx > m_ref + kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - mx);
        l *= alpha;
        m_ref = mx;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O is rescaled in place once the previous PV finished writing it
        if (!(ok = warp_wait_bar(bar_o(X), (j - 1) & 1, abort_flag, p.err))) break;
        tc_fence_after();
        uint32_t o[32];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld_32x32b_x32(o_addr + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(o_addr + c * 32, o);
        }
        tmem_st_wait();
      }
      // P = 2^(s * scale_log2 - m): one FFMA + one exp2 per score.  bf16 pairs overwrite the first
      // half of S's columns: half h's pairs land on columns [32h, 32h + 32), all of which hold
      // scores already read into registers.
      const float neg_m = -m_ref;
      float s8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) s8[k] = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t t[2][32];
        tmem_ld_32x32b_x32(s_addr + half * 64, t[0]);
        tmem_ld_32x32b_x32(s_addr + half * 64 + 32, t[1]);
        tmem_ld_wait();
        if (diag) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (half * 64 + c > r) t[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // 16 scores -> 8 packed columns per store
          uint32_t packed[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int c0 = g * 16 + 2 * i, c1 = c0 + 1;
            const float e0 = ex2_mixed<kFma>(fmaf(__uint_as_float(t[c0 >> 5][c0 & 31]), p.scale_log2, neg_m), c0);
            const float e1 = ex2_mixed<kFma>(fmaf(__uint_as_float(t[c1 >> 5][c1 & 31]), p.scale_log2, neg_m), c1);
            s8[c0 & 7] += e0;
            s8[c1 & 7] += e1;
            packed[i] = pack_bf16x2(e0, e1);
          }
          tmem_st_32x32b_x8(s_addr + half * 32 + g * 8, packed);
        }
      }
      const float sum = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
      tmem_st_wait();
      l += sum;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p(X));
    }
    if (ok && warp_wait_bar(bar_o(X), jmax & 1, abort_flag, p.err)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int q = q0 + X * kTile + r;
      __nv_bfloat16* orow = p.o + static_cast<long long>(row_base + q) * p.o_stride + h * kTile;
      uint32_t t[32];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld_32x32b_x32(o_addr + c * 32, t);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(t[8 * i + 0]) * inv, __uint_as_float(t[8 * i + 1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(t[8 * i + 2]) * inv, __uint_as_float(t[8 * i + 3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(t[8 * i + 4]) * inv, __uint_as_float(t[8 * i + 5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(t[8 * i + 6]) * inv, __uint_as_float(t[8 * i + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * i) = u;
        }
      }
      p.lse[(static_cast<long long>(b) * p.Hq + h) * p.S + q] = (m_ref + __log2f(l)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Exponentials per 8 score columns evaluated on the FMA pipe (ex2_fma) by default.  Measured on
// B200 at B=2 S=4096 (forward / backward TFLOP/s for shares 0..3): 797/585, 768/581, 751/572,
// 732/561 -- with the softmax's dependency chains broken up the MUFU unit is not the limit, so
// every exponential stays on MUFU; the other shares remain selectable for tuning.
constexpr int kDefaultFmaShare = 0;

template <int kFma>
int launch_fwd(int grid, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FwdParams& p,
               cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_sm100_kernel<kFma>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr = true;
  }
  attn_fwd_sm100_kernel<kFma><<<grid, kThreads, kSmem, stream>>>(tq, tk, tv, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

// Returns 1 when the shape is not handled by this kernel (the caller uses the mma.sync path).
// ``variant``: exponentials per 8 score columns on the FMA pipe (0-3), or -1 for the default.
int attention_fwd_sm100(const AttnArgs& a, int D, int* err, cudaStream_t stream, int variant) {
  if (D != 128 || !a.causal || a.S % 256 != 0 || a.Hq % a.Hkv != 0) return 1;
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
       reinterpret_cast<uintptr_t>(a.o)) & 15)
    return 1;
  if ((a.q_stride | a.k_stride | a.v_stride | a.o_stride) & 7) return 1;
  const long long T = static_cast<long long>(a.B) * a.S;
  CUtensorMap tq, tk, tv;
  if (make_tmap_bf16_2d(&tq, a.q, static_cast<uint64_t>(a.Hq) * 128, T, a.q_stride, 64, 128)) return -20;
  if (make_tmap_bf16_2d(&tk, a.k, static_cast<uint64_t>(a.Hkv) * 128, T, a.k_stride, 64, 128)) return -21;
  if (make_tmap_bf16_2d(&tv, a.v, static_cast<uint64_t>(a.Hkv) * 128, T, a.v_stride, 64, 128)) return -22;
  FwdParams p{reinterpret_cast<__nv_bfloat16*>(a.o), a.o_stride, a.lse, a.B, a.S, a.Hq, a.Hkv,
              a.scale * 1.4426950408889634f, err};
  const int grid = (a.S / 256) * a.Hq * a.B;
  switch (variant < 0 ? kDefaultFmaShare : variant) {
    case 0: return launch_fwd<0>(grid, tq, tk, tv, p, stream);
    case 1: return launch_fwd<1>(grid, tq, tk, tv, p, stream);
    case 2: return launch_fwd<2>(grid, tq, tk, tv, p, stream);
    case 3: return launch_fwd<3>(grid, tq, tk, tv, p, stream);
    default: return -23;
  }
}

}  // namespace rb
