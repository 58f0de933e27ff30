// Persistent warp-specialised bf16 GEMM on the 5th-generation tensor cores (tcgen05 / TMEM).
//
//   D[m, n] = alpha * sum_k A(m, k) * B(n, k)          (+ epilogue: residual / accumulate)
//
// A and B are each either K-major (row of the operand contiguous along k) or MN-major
// (contiguous along m / n), so a linear layer's forward (x W^T), dgrad (dy W) and wgrad
// (dy^T x) all run without a transpose.
//
// Roles per CTA (one CTA per SM, grid = min(#tiles, #SMs), static round-robin over tiles):
//   warp 0      : TMA producer, STAGES-deep ring of (A, B) tiles, 128B swizzle
//   warp 1      : TMEM allocator and single-thread tcgen05.mma issuer
//   warps 2..5  : epilogue, tcgen05.ld of the accumulator rows owned by the warp's lane
//                 quadrant, fused scale / residual / fp32 accumulate, vector stores
// The accumulator is double buffered in TMEM (2 x BN columns) so the epilogue of tile i
// overlaps the MMAs of tile i+1.
//
// This file is new work: the reference framework has no GEMM of its own (its compute
// validation probe `resihp/detect/validation.py:17-31` calls torch.matmul).
#include <cuda.h>
#include <cstring>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "sm100.cuh"
#include "tmap.h"

namespace rb {

enum : int { kEpiBF16 = 0, kEpiF32 = 1, kEpiF32Acc = 2, kEpiBF16Res = 3, kEpiScatterBF16 = 4 };

constexpr int kMaxTP = 8;
constexpr int kAgSegCols = 512;  // columns per all-gather copy unit (a multiple of the 64-column k-block)

struct GemmArgs {
  int M, N, K;
  void* D;
  long long ldd;
  const __nv_bfloat16* R;
  long long ldr;
  float alpha;
  int* err;
  // kEpiScatterBF16 (GEMM -> reduce-scatter): output rows [q * rs_rows, (q + 1) * rs_rows) are
  // stored as bf16 into rank q's receive buffer, slot `rs_slot` ([world][rs_rows][N] elements).
  int rs_slot, rs_rows;
  void* rs_dst[kMaxTP];
  // all-gather -> GEMM: A's rows come in `ag_world` chunks of `ag_chunk_rows`; this rank owns
  // chunk `ag_self` (already in place in `ag_dst`); the kernel's copy warps pull the other chunks
  // from `ag_src[c]` into `ag_dst` in units of 128 rows x `ag_kseg` columns, taken from the work
  // counter `ag_ready[0]`, and publish each finished unit in its flag `ag_ready[1 + unit]`.
  int ag_world, ag_self, ag_chunk_rows, ag_kseg;
  const void* ag_src[kMaxTP];
  void* ag_dst;
  int* ag_ready;
  const int* abort_word;
  // split-K of the CTA-pair kernel: `splits` (1 or 2) work units per output tile, each over its
  // share of the k-blocks.  Every unit's epilogue warp stores its 32 x 256 fp32 partial into its
  // own workspace slot and counts itself on the tile's (CTA, warp) counter; the last to arrive
  // adds the slots in a fixed order and runs the epilogue (so the result does not depend on which
  // unit finishes first).
  int splits;
  float* split_ws;
  int* split_cnt;
  // split only the tiles past the first `split_full` (the partial last wave): those run as
  // `splits` shares each, the earlier ones whole
  int split_full;
};

// One work unit of the CTA-pair kernel: tiles [0, full) whole, then the tail tiles' k shares in
// share-major order (every tail tile's first share before any second share).  `tail_idx` < 0 for
// a whole tile.
struct PairUnit {
  int tile, share, kb_lo, kb_hi, tail_idx;
};

__device__ __forceinline__ PairUnit pair_unit(int u, int num_tiles, int full, int splits, int kblocks) {
  PairUnit w;
  if (u < full || splits == 1) {
    w.tile = u;
    w.share = 0;
    w.kb_lo = 0;
    w.kb_hi = kblocks;
    w.tail_idx = -1;
    return w;
  }
  const int tail = num_tiles - full;
  const int v = u - full;
  const int kb_share = (kblocks + splits - 1) / splits;
  w.tail_idx = v % tail;
  w.tile = full + w.tail_idx;
  w.share = v / tail;
  w.kb_lo = w.share * kb_share;
  w.kb_hi = min(kblocks, w.kb_lo + kb_share);
  return w;
}

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // 64 bf16 = 128 B = one swizzle row
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  static constexpr int STAGING_BYTES = 4 * 4096;  // scatter epilogue: 32 rows x 64 bf16 per warp
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + STAGING_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 192;
  static constexpr int GROUP_M = 16;
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& mb,
                                            int& nb) {
  const int per_group = group_m * num_n;
  const int g = tile / per_group;
  const int first_m = g * group_m;
  const int gsize = min(num_m - first_m, group_m);
  const int r = tile - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// Epilogue of one 32-column chunk of one accumulator row: scale, optional residual / fp32
// accumulate, vector stores (column tail handled scalar).
template <int EPI>
__device__ __forceinline__ void store_chunk(const uint32_t (&r)[32], int row, int col0, const GemmArgs& p) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
  const bool full = (col0 + 32 <= p.N);
  if (EPI == kEpiScatterBF16) {
    const int q = row / p.rs_rows;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.rs_dst[q]) +
                         (static_cast<long long>(p.rs_slot) * p.rs_rows + (row - q * p.rs_rows)) * p.N + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 u;
        u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
        u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        *reinterpret_cast<uint4*>(dst + 8 * j) = u;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) dst[j] = __float2bfloat16_rn(v[j]);
    }
    return;
  }
  if (EPI == kEpiBF16 || EPI == kEpiBF16Res) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd + col0;
    if (EPI == kEpiBF16Res) {
      const __nv_bfloat16* res = p.R + row * p.ldr + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 u = *reinterpret_cast<const uint4*>(res + 8 * j);
          float2 f0 = unpack_bf16x2(u.x), f1 = unpack_bf16x2(u.y), f2 = unpack_bf16x2(u.z),
                 f3 = unpack_bf16x2(u.w);
          v[8 * j + 0] += f0.x; v[8 * j + 1] += f0.y; v[8 * j + 2] += f1.x; v[8 * j + 3] += f1.y;
          v[8 * j + 4] += f2.x; v[8 * j + 5] += f2.y; v[8 * j + 6] += f3.x; v[8 * j + 7] += f3.y;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) v[j] += __bfloat162float(res[j]);
      }
    }
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 u;
        u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
        u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        *reinterpret_cast<uint4*>(dst + 8 * j) = u;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) dst[j] = __float2bfloat16_rn(v[j]);
    }
  } else {
    float* dst = reinterpret_cast<float*>(p.D) + row * p.ldd + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        if (EPI == kEpiF32Acc) {
          const float4 old = *reinterpret_cast<const float4*>(dst + 4 * j);
          o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
        }
        *reinterpret_cast<float4*>(dst + 4 * j) = o;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) dst[j] = (EPI == kEpiF32Acc) ? dst[j] + v[j] : v[j];
    }
  }
}

// lane 0 waits, the whole warp learns the outcome
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    GemmArgs p) {
  using C = GemmCfg<BN>;
  constexpr int BM = C::BM, BK = C::BK, STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* staging = sB + STAGES * C::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + 2 + a]); };
  const uint32_t final_bar = smem_u32(&bars[2 * STAGES + 4]);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;      // stages with a load in flight at some point
      uint32_t issued_parity = 0;    // parity of the last load issued into each stage
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, C::GROUP_M, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
          const uint32_t a_dst = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * C::B_BYTES);
          if (!A_MN) {
            tma_load_2d(a_dst, &tmA, fb, kb * BK, mb * BM);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 8192, &tmA, fb, mb * BM + 64 * j, kb * BK);
          }
          if (!B_MN) {
            tma_load_2d(b_dst, &tmB, fb, kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, fb, nb * BN + 64 * j, kb * BK);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // Drain: every load this thread issued must have landed before the CTA exits.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s))
          mbar_wait(full_bar(s), (issued_parity >> s) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, true, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), aphase ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? make_smem_desc(a_base + k * 2048, 8192, 1024, kSwizzle128B)
                                     : make_smem_desc(a_base + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = B_MN ? make_smem_desc(b_base + k * 2048, 8192, 1024, kSwizzle128B)
                                     : make_smem_desc(b_base + k * 32, 16, 1024, kSwizzle128B);
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) aphase ^= 1;
      }
      // Every MMA issued by this thread completes before TMEM is released.
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t aphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, C::GROUP_M, mb, nb);
      if (!warp_wait(tfull_bar(acc), aphase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
      if constexpr (EPI == kEpiScatterBF16) {
        // Stores to another GPU's memory: stage 32 rows x 64 columns per warp in shared memory so
        // that each warp instruction writes four whole 128-byte row segments (8 KB per flush),
        // instead of 32 scattered 16-byte pieces.
        uint8_t* st = staging + (warp - 2) * 4096;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          uint32_t r0[32], r1[32];
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c * 32;
          tmem_ld_32x32b_x32(taddr, r0);
          tmem_ld_32x32b_x32(taddr + 32, r1);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // 16-byte chunk j of this lane's 128-byte row, XOR-swizzled
            const uint32_t* src = j < 4 ? r0 + 8 * j : r1 + 8 * (j - 4);
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(src[0]) * p.alpha, __uint_as_float(src[1]) * p.alpha);
            u.y = pack_bf16x2(__uint_as_float(src[2]) * p.alpha, __uint_as_float(src[3]) * p.alpha);
            u.z = pack_bf16x2(__uint_as_float(src[4]) * p.alpha, __uint_as_float(src[5]) * p.alpha);
            u.w = pack_bf16x2(__uint_as_float(src[6]) * p.alpha, __uint_as_float(src[7]) * p.alpha);
            *reinterpret_cast<uint4*>(st + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = i * 4 + (lane >> 3);  // row within the warp's 32
            const int seg = lane & 7;
            const int grow = mb * BM + q * 32 + rr;
            const int gcol = nb * BN + c * 32 + seg * 8;
            if (grow < p.M && gcol < p.N) {
              const uint4 u = *reinterpret_cast<const uint4*>(st + rr * 128 + ((seg ^ (rr & 7)) << 4));
              const int owner = grow / p.rs_rows;
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.rs_dst[owner]) +
                                   (static_cast<long long>(p.rs_slot) * p.rs_rows + (grow - owner * p.rs_rows)) * p.N +
                                   gcol;
              *reinterpret_cast<uint4*>(dst) = u;
            }
          }
          __syncwarp();
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c * 32, r);
          tmem_ld_wait();
          const int col0 = nb * BN + c * 32;
          if (!row_ok || col0 >= p.N) continue;
          store_chunk<EPI>(r, row, col0, p);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) aphase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- all-gather -> GEMM
// Column-parallel layer with sequence-parallel input: Y = AllGather_rows(X) @ W^T in one
// persistent launch.  Warps 0-5 are the GEMM above (128 x 256 tiles); warps 6-9 pull the other
// ranks' row chunks of X over NVLink into this rank's gather buffer (16-byte peer loads).  The
// remote rows are cut into units of 128 rows x `ag_kseg` columns, enumerated chunk by chunk in
// the rotated order self+1, self+2, ...; each CTA's copy warps take the next unit from a global
// work counter, copy it and publish it with a release flag.  Tiles are visited in the same
// rotated order starting with this rank's own chunk, so the MMAs of early chunks overlap the
// transfer of later ones; before loading A's k-block the TMA producer waits (bounded, acquire +
// proxy fence) for the flag of the unit holding it.  A unit is only ever awaited after some
// running CTA claimed it or while unclaimed units remain for the copy warps of running CTAs, so
// the waits make progress however many CTAs are resident: the launch is an ordinary one and may
// share the GPU with other kernels (NCCL's included).  The caller orders the launch after the
// peers wrote their chunks (a bounded cross-GPU barrier) and before they overwrite them.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int EPI, bool B_MN>
__global__ void __launch_bounds__(320, 1)
    gemm_ag_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  using C = GemmCfg<256>;
  constexpr int BM = C::BM, BN = 256, BK = C::BK, STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * C::B_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* unit_slot = reinterpret_cast<int*>(tmem_slot + 2);  // copy warps: the unit being copied
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + 2 + a]); };
  const uint32_t final_bar = smem_u32(&bars[2 * STAGES + 4]);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;
  const int mb_per_chunk = p.ag_chunk_rows / BM;
  const int rot = p.ag_self * mb_per_chunk;  // visit this rank's own chunk first
  const int nseg = (p.K + p.ag_kseg - 1) / p.ag_kseg;
  auto coords = [&](int tile, int& mb, int& nb) {
    tile_coords(tile, num_m, num_n, C::GROUP_M, mb, nb);
    mb = (mb + rot) % num_m;
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        coords(tile, mb, nb);
        const bool remote = mb / mb_per_chunk != p.ag_self;
        int seg_ready = remote ? -1 : nseg;  // k-segments of this row block known to be in place
        for (int kb = 0; kb < kblocks; ++kb) {
          const int seg = kb * BK / p.ag_kseg;
          if (seg > seg_ready) {
            const int* flag = p.ag_ready + 1 + mb * nseg + seg;
            const uint64_t t0 = globaltimer();
            while (ld_acquire_gpu(flag) == 0) {
              if (*abort_flag || (p.abort_word != nullptr && *reinterpret_cast<const volatile int*>(p.abort_word))) {
                ok = false;
                break;
              }
              if (globaltimer() - t0 > kWaitBudgetNs) {
                *abort_flag = 1;
                record_error(p.err, kErrPeerTimeout);
                ok = false;
                break;
              }
              __nanosleep(64);
            }
            if (!ok) break;
            fence_proxy_async_global();  // generic-proxy writes of the copy warps -> TMA reads
            seg_ready = seg;
          }
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
          tma_load_2d(smem_u32(sA + stage * C::A_BYTES), &tmA, fb, kb * BK, mb * BM);
          if (!B_MN) {
            tma_load_2d(smem_u32(sB + stage * C::B_BYTES), &tmB, fb, kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(smem_u32(sB + stage * C::B_BYTES) + j * 8192, &tmB, fb, nb * BN + 64 * j, kb * BK);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) *abort_flag = 1;
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_parity >> s) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, true, false, B_MN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, aphase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), aphase ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d_tmem, make_smem_desc(a_base + k * 32, 16, 1024, kSwizzle128B),
                     B_MN ? make_smem_desc(b_base + k * 2048, 8192, 1024, kSwizzle128B)
                          : make_smem_desc(b_base + k * 32, 16, 1024, kSwizzle128B),
                     idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) aphase ^= 1;
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, p.err, 200000000ull);
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    int acc = 0;
    uint32_t aphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      coords(tile, mb, nb);
      if (!warp_wait(tfull_bar(acc), aphase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + c * 32, r);
        tmem_ld_wait();
        const int col0 = nb * BN + c * 32;
        if (!row_ok || col0 >= p.N) continue;
        store_chunk<EPI>(r, row, col0, p);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) aphase ^= 1;
    }
  } else {
    // ------------------------------------------------------------ copy warps 6..9
    const int t = threadIdx.x - 192;  // 0..127
    const int remote_blocks = (p.ag_world - 1) * mb_per_chunk;
    const int units = remote_blocks * nseg;
    for (;;) {
      if (t == 0) *unit_slot = atomicAdd(p.ag_ready, 1);
      named_bar_sync(1, 128);
      const int u = *unit_slot;
      named_bar_sync(1, 128);  // every copy thread read the unit before it is replaced
      if (u >= units) break;
      const int rb = u / nseg, seg = u - rb * nseg;
      const int c = (p.ag_self + 1 + rb / mb_per_chunk) % p.ag_world;
      const int mb = c * mb_per_chunk + rb % mb_per_chunk;
      const int row0 = mb * BM - c * p.ag_chunk_rows;  // first row of the unit within chunk c
      const int col0 = seg * p.ag_kseg;
      const int gpr = (min(p.K - col0, p.ag_kseg)) / 8;  // 16-byte granules per row of the unit
      const int total = BM * gpr;
      const uint4* src = reinterpret_cast<const uint4*>(p.ag_src[c]);
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.ag_dst) +
                                            static_cast<long long>(c) * p.ag_chunk_rows * p.K * 2);
      const long long ld16 = p.K / 8;  // granules per row of the matrix
      for (int i = t; i < total; i += 128 * 8) {
        uint4 v[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const int g = i + w * 128;
          if (g < total) {
            const int r = g / gpr, q = g - r * gpr;
            v[w] = __ldcv(src + (row0 + r) * ld16 + col0 / 8 + q);
          }
        }
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const int g = i + w * 128;
          if (g < total) {
            const int r = g / gpr, q = g - r * gpr;
            dst[(row0 + r) * ld16 + col0 / 8 + q] = v[w];
          }
        }
      }
      __threadfence();
      fence_proxy_async_global();  // this thread's generic writes -> the consumers' TMA (async proxy) reads
      named_bar_sync(1, 128);
      if (t == 0) st_release_gpu(p.ag_ready + 1 + mb * nseg + seg, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- CTA-pair kernel
// Same roles, but a cluster of two CTAs computes one 256 x 256 tile with cta_group::2 MMAs:
// CTA r holds rows [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B
// tile, and its TMEM receives rows [128 r, 128 r + 128) of D (all 256 columns).  Per k-block each
// CTA loads 32 KB instead of 48 KB, so 6 stages fit and L2->SM traffic per FLOP drops by a third.
//   * both CTAs' TMA loads count on the leader's full barrier (the leader expects both halves);
//   * the leader issues the MMAs and commits separately to each CTA's empty / accumulator-full
//     barriers (no multicast);
//   * epilogue warps of both CTAs release the accumulator on the leader's barrier (8 arrivals);
//   * optional split-K of the tiles of the partial last wave (`PairUnit`): full waves run whole
//     tiles, each tail tile runs as up to 4 k shares whose fp32 partials the last-arriving share
//     adds in a fixed order (deterministic) before the epilogue.
// Epilogues the CTA-pair kernel writes with TMA (shared-memory staging, tile store or fp32
// reduce-add) when its ring leaves room for the staging buffers.
template <int EPI>
constexpr bool pair_tma_epi() {
  return EPI == kEpiBF16 || EPI == kEpiF32 || EPI == kEpiF32Acc;
}

template <int kStages, int kBN = 256, int EPI = kEpiBF16>
struct PairCfg {
  static constexpr int BM = 128;  // rows per CTA (the pair covers 256)
  static constexpr int BN = kBN;  // columns of the pair's tile (256, or 128 for more tiles per wave)
  static constexpr int BNH = kBN / 2;  // B rows held per CTA
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BNH * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = kStages;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  // TMA epilogue: per epilogue warp two 32 x 32 staging tiles of the output type
  static constexpr int OUT_BYTES = (EPI == kEpiF32 || EPI == kEpiF32Acc) ? 4 : 2;
  static constexpr int STG_TILE = 32 * 32 * OUT_BYTES;
  static constexpr int BASE_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARS * 8 + 16;
  static constexpr bool TMA_EPI = pair_tma_epi<EPI>() && BASE_BYTES + 8 * STG_TILE <= 232448;
  static constexpr int STG_BYTES = TMA_EPI ? 8 * STG_TILE : 0;
  static constexpr int SMEM_BYTES = BASE_BYTES + STG_BYTES;
  static constexpr int THREADS = 192;
  static constexpr int GROUP_M = 8;  // in 256-row pair tiles
  static_assert(SMEM_BYTES <= 232448, "over the 227 KB of dynamic shared memory a CTA may have");
};

template <bool A_MN, bool B_MN, int EPI, int kStages, int kBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_bf16_sm100_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmD, GemmArgs p) {
  using C = PairCfg<kStages, kBN, EPI>;
  constexpr int BM = C::BM, BK = C::BK, STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* stg = sB + STAGES * C::B_BYTES;  // TMA epilogue staging (C::STG_BYTES)
  uint64_t* bars = reinterpret_cast<uint64_t*>(stg + C::STG_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * STAGES + 2 + a]); };
  const uint32_t final_bar = smem_u32(&bars[2 * STAGES + 4]);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const bool leader = cta == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (p.M + 2 * BM - 1) / (2 * BM);
  const int num_n = (p.N + C::BN - 1) / C::BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int splits = p.splits > 1 ? min(p.splits, 4) : 1;
  const int full = splits > 1 ? min(max(p.split_full, 0), num_tiles) : num_tiles;
  const int num_units = full + splits * (num_tiles - full);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      for (int u = pair; u < num_units && !*abort_flag; u += num_pairs) {
        const PairUnit w = pair_unit(u, num_tiles, full, splits, kblocks);
        const int tile = w.tile, kb_lo = w.kb_lo, kb_hi = w.kb_hi;
        int mb, nb;
        tile_coords(tile, num_m, num_n, C::GROUP_M, mb, nb);
        const int m0 = mb * 2 * BM + static_cast<int>(cta) * BM;
        const int n0 = nb * C::BN + static_cast<int>(cta) * C::BNH;
        bool ok = true;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = full_bar(stage);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * C::STAGE_BYTES);
          const uint32_t fb = mapa_shared(fb_local, 0);
          const uint32_t a_dst = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * C::B_BYTES);
          if (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a_dst + j * 8192, &tmA, fb, m0 + 64 * j, kb * BK);
          }
          if (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, fb, kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < C::BNH / 64; ++j) tma_load_2d_pair(b_dst + j * 8192, &tmB, fb, n0 + 64 * j, kb * BK);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // Drain (leader: its full barriers count both CTAs' loads; the peer's loads of a stage
      // complete before the leader's barrier phase does).
      if (leader)
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(full_bar(s), (issued_parity >> s) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_f16(2 * BM, C::BN, true, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      for (int u = pair; u < num_units; u += num_pairs) {
        const PairUnit w = pair_unit(u, num_tiles, full, splits, kblocks);
        const int kb_lo = w.kb_lo, kb_hi = w.kb_hi;
        if (!mbar_wait(tempty_bar(acc), aphase ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BN;
        bool ok = true;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? make_smem_desc(a_base + k * 2048, 8192, 1024, kSwizzle128B)
                                     : make_smem_desc(a_base + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = B_MN ? make_smem_desc(b_base + k * 2048, 8192, 1024, kSwizzle128B)
                                     : make_smem_desc(b_base + k * 32, 16, 1024, kSwizzle128B);
            umma_f16_pair(d_tmem, ad, bd, idesc, (kb != kb_lo || k != 0) ? 1u : 0u);
          }
          umma_commit_pair(empty_bar(stage));
          umma_commit_pair(mapa_shared(empty_bar(stage), 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(acc));
        umma_commit_pair(mapa_shared(tfull_bar(acc), 1));
        acc ^= 1;
        if (acc == 0) aphase ^= 1;
      }
      umma_commit_pair(final_bar);
      mbar_wait(final_bar, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    const uint32_t release = leader ? 0u : mapa_shared(tempty_bar(0), 0);  // peer: leader's barrier
    int acc = 0;
    uint32_t aphase = 0;
    int stg_buf = 0;
    for (int u = pair; u < num_units; u += num_pairs) {
      const PairUnit w = pair_unit(u, num_tiles, full, splits, kblocks);
      const int tile = w.tile, share = w.share;
      const bool split_unit = w.tail_idx >= 0;
      int mb, nb;
      tile_coords(tile, num_m, num_n, C::GROUP_M, mb, nb);
      if (!warp_wait(tfull_bar(acc), aphase, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = mb * 2 * BM + static_cast<int>(cta) * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * C::BN;
      // workspace slots of this (tail tile, CTA, warp): `splits` consecutive 32 x BN fp32 blocks
      const long long slot0 =
          static_cast<long long>((max(w.tail_idx, 0) * 2 + static_cast<int>(cta)) * 4 + q) * splits;
      if (!split_unit && C::TMA_EPI) {
        // 32 x 32 output boxes through two staging tiles per warp: each lane writes its row into
        // the tile, the tile goes to global memory as one TMA store (fp32 accumulate: TMA
        // reduce-add in L2); TMA clips rows past M and columns past N.
        const int row0 = mb * 2 * BM + static_cast<int>(cta) * BM + q * 32;
#pragma unroll 1
        for (int c = 0; c < C::BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, r);
          tmem_ld_wait();
          const int col0 = nb * C::BN + c * 32;
          if (row0 >= p.M || col0 >= p.N) continue;
          uint8_t* tile = stg + (q * 2 + stg_buf) * C::STG_TILE;
          if (lane == 0) bulk_wait_group_read<1>();  // this tile's previous store has read it
          __syncwarp();
          if constexpr (C::OUT_BYTES == 2) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              w[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * p.alpha, __uint_as_float(r[2 * i + 1]) * p.alpha);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<uint4*>(tile + lane * 64 + j * 16) =
                  make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(tile + lane * 128 + j * 16) =
                  make_float4(__uint_as_float(r[4 * j]) * p.alpha, __uint_as_float(r[4 * j + 1]) * p.alpha,
                              __uint_as_float(r[4 * j + 2]) * p.alpha, __uint_as_float(r[4 * j + 3]) * p.alpha);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == kEpiF32Acc) tma_reduce_add_2d(&tmD, smem_u32(tile), col0, row0);
            else tma_store_2d(&tmD, smem_u32(tile), col0, row0);
            bulk_commit_group();
          }
          stg_buf ^= 1;
        }
      } else if (!split_unit) {
#pragma unroll 1
        for (int c = 0; c < C::BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, r);
          tmem_ld_wait();
          const int col0 = nb * C::BN + c * 32;
          if (!row_ok || col0 >= p.N) continue;
          store_chunk<EPI>(r, row, col0, p);
        }
      } else {
        // this unit's partial -> its slot, column-major (each store is one coalesced 128-byte row)
        float* mine = p.split_ws + (slot0 + share) * (32 * C::BN);
#pragma unroll 1
        for (int c = 0; c < C::BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) mine[(c * 32 + i) * 32 + lane] = __uint_as_float(r[i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(tempty_bar(acc));
        else mbar_arrive_cluster(release + acc * 8);
      }
      if (split_unit) {
        // the accumulator is released already; the unit that arrives last reduces the slots
        __threadfence();
        __syncwarp();
        int* cnt = p.split_cnt + (w.tail_idx * 2 + static_cast<int>(cta)) * 4 + q;
        int last = 0;
        if (lane == 0) last = atomicAdd(cnt, 1) == splits - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          // shares added in a fixed order; every share's 32 loads of a chunk are independent and in
          // flight together (one load per round trip made an earlier version ~10x slower)
          const float* s0 = p.split_ws + slot0 * (32 * C::BN);
#pragma unroll 1
          for (int c = 0; c < C::BN / 32; ++c) {
            const int col0 = nb * C::BN + c * 32;
            float a0[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) a0[i] = __ldcg(s0 + (c * 32 + i) * 32 + lane);
            for (int sh = 1; sh < splits; ++sh) {
              float b[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) b[i] = __ldcg(s0 + sh * (32 * C::BN) + (c * 32 + i) * 32 + lane);
#pragma unroll
              for (int i = 0; i < 32; ++i) a0[i] += b[i];
            }
            uint32_t r[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(a0[i]);
            if (row_ok && col0 < p.N) store_chunk<EPI>(r, row, col0, p);
          }
          if (lane == 0) *cnt = 0;  // ready for the next launch (the host also clears it first)
        }
      }
      acc ^= 1;
      if (acc == 0) aphase ^= 1;
    }
    if (C::TMA_EPI && lane == 0) bulk_wait_group_all();  // this warp's stores have landed
  }

  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs may still read its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (h) fn = reinterpret_cast<EncodeTiledFn>(dlsym(h, "cuTensorMapEncodeTiled"));
  });
  return fn;
}

int make_tmap_2d_sw128(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes, const void* ptr, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

int make_tmap_2d_plain(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes, const void* ptr, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

// 2-D bf16 tensor map, 128B swizzle: `inner` contiguous elements per row, `outer` rows.
int make_tmap_bf16_2d(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int num_sms,
                       cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kern = gemm_bf16_sm100<BN, A_MN, B_MN, EPI>;
  static bool attr_set = false;  // per instantiation; attribute is per function and device-agnostic
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  const int tiles = ((a.M + C::BM - 1) / C::BM) * ((a.N + BN - 1) / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  kern<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(ta, tb, a);
  return static_cast<int>(cudaGetLastError());
}

template <bool A_MN, bool B_MN, int EPI, int kStages, int kBN>
static int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int num_sms,
                            cudaStream_t stream) {
  using C = PairCfg<kStages, kBN, EPI>;
  auto kern = gemm_bf16_sm100_pair<A_MN, B_MN, EPI, kStages, kBN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  CUtensorMap td;  // output boxes of 32 x 32 for the TMA epilogue (unused otherwise)
  std::memset(&td, 0, sizeof(td));
  if (C::TMA_EPI) {
    const bool f32 = C::OUT_BYTES == 4;
    if (int rc = make_tmap_2d_plain(&td, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                    C::OUT_BYTES, a.D, a.N, a.M, a.ldd, 32, 32))
      return -100 - rc;
  }
  const int tiles = ((a.M + 2 * C::BM - 1) / (2 * C::BM)) * ((a.N + C::BN - 1) / C::BN);
  int pairs = num_sms / 2;
  const int full = a.splits > 1 ? a.split_full : tiles;
  const int units = full + (a.splits > 1 ? a.splits : 1) * (tiles - full);
  if (units < pairs) pairs = units;
  kern<<<2 * pairs, C::THREADS, C::SMEM_BYTES, stream>>>(ta, tb, td, a);
  return static_cast<int>(cudaGetLastError());
}

template <int EPI, int kStages, int kBN>
static int dispatch_major_pair_stages(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                                      const GemmArgs& a, int num_sms, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_gemm_pair<false, false, EPI, kStages, kBN>(ta, tb, a, num_sms, s);
  if (!a_mn && b_mn) return launch_gemm_pair<false, true, EPI, kStages, kBN>(ta, tb, a, num_sms, s);
  if (a_mn && !b_mn) return launch_gemm_pair<true, false, EPI, kStages, kBN>(ta, tb, a, num_sms, s);
  return launch_gemm_pair<true, true, EPI, kStages, kBN>(ta, tb, a, num_sms, s);
}

// `stages`: depth of the operand ring (6 by default; 7 fills the 227 KB of shared memory);
// `bn`: pair tile width, 256, or 128 (8 stages) for twice the tiles per wave
template <int EPI>
static int dispatch_major_pair(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                               const GemmArgs& a, int num_sms, cudaStream_t s, int stages, int bn) {
  if (bn == 128) return dispatch_major_pair_stages<EPI, 8, 128>(a_mn, b_mn, ta, tb, a, num_sms, s);
  if (stages == 7) return dispatch_major_pair_stages<EPI, 7, 256>(a_mn, b_mn, ta, tb, a, num_sms, s);
  return dispatch_major_pair_stages<EPI, 6, 256>(a_mn, b_mn, ta, tb, a, num_sms, s);
}

template <int BN, int EPI>
static int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmArgs& a, int num_sms, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_gemm<BN, false, false, EPI>(ta, tb, a, num_sms, s);
  if (!a_mn && b_mn) return launch_gemm<BN, false, true, EPI>(ta, tb, a, num_sms, s);
  if (a_mn && !b_mn) return launch_gemm<BN, true, false, EPI>(ta, tb, a, num_sms, s);
  return launch_gemm<BN, true, true, EPI>(ta, tb, a, num_sms, s);
}

template <int BN>
static int dispatch_epi(int epi, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GemmArgs& a, int num_sms, cudaStream_t s) {
  switch (epi) {
    case kEpiBF16: return dispatch_major<BN, kEpiBF16>(a_mn, b_mn, ta, tb, a, num_sms, s);
    case kEpiF32: return dispatch_major<BN, kEpiF32>(a_mn, b_mn, ta, tb, a, num_sms, s);
    case kEpiF32Acc: return dispatch_major<BN, kEpiF32Acc>(a_mn, b_mn, ta, tb, a, num_sms, s);
    case kEpiBF16Res: return dispatch_major<BN, kEpiBF16Res>(a_mn, b_mn, ta, tb, a, num_sms, s);
  }
  return -2;
}

// Y[M, N] = AllGather(X)[M, K] @ W[N, K]^T with the gather fused (see gemm_ag_sm100).
// `x_full` is this rank's [M, K] gather buffer (its own chunk already in place), `x_src[c]` the
// address of chunk c in rank c's buffer (peer memory), `ready` `world` zeroed ints.
int gemm_ag_bf16(const void* x_full, const void* const* x_src, int world, int self, int chunk_rows, const void* W,
                 bool w_mn, void* Y, int M, int N, int K, int* ready, const int* abort_word, int* err, int num_sms,
                 cudaStream_t stream) {
  if (world < 1 || world > kMaxTP || chunk_rows % 128 || M != chunk_rows * world || K % 8 || N % 8) return -3;
  if ((reinterpret_cast<uintptr_t>(x_full) | reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(Y)) & 15)
    return -4;
  for (int c = 0; c < world; ++c)
    if (reinterpret_cast<uintptr_t>(x_src[c]) & 15) return -4;
  CUtensorMap ta, tb;
  if (int rc = make_tmap_bf16_2d(&ta, x_full, K, M, K, 64, 128)) return -100 - rc;
  // W is [N, K] (K-major) or, with w_mn, [K, N] (B(n, k) = W[k * N + n])
  if (int rc = w_mn ? make_tmap_bf16_2d(&tb, W, N, K, N, 64, 64) : make_tmap_bf16_2d(&tb, W, K, N, K, 64, 256))
    return -100 - rc;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.D = Y; a.ldd = N; a.alpha = 1.f; a.err = err;
  a.ag_world = world; a.ag_self = self; a.ag_chunk_rows = chunk_rows; a.ag_kseg = kAgSegCols;
  for (int c = 0; c < world; ++c) a.ag_src[c] = x_src[c];
  a.ag_dst = const_cast<void*>(x_full);
  a.ag_ready = ready;
  a.abort_word = abort_word;
  using C = GemmCfg<256>;
  auto kern = w_mn ? gemm_ag_sm100<kEpiBF16, true> : gemm_ag_sm100<kEpiBF16, false>;
  static bool attr[2] = {false, false};
  if (!attr[w_mn]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr[w_mn] = true;
  }
  kern<<<num_sms, 320, C::SMEM_BYTES, stream>>>(ta, tb, a);
  return static_cast<int>(cudaGetLastError());
}

int gemm_ag_ready_words(int M, int K) { return 1 + (M / 128) * ((K + kAgSegCols - 1) / kAgSegCols); }

// Partial products of a row-parallel layer, scattered for a reduce-scatter: rows
// [q * (M / world), (q + 1) * (M / world)) of X[M, K] @ W[N, K]^T are stored (bf16) into
// `recv[q]` (rank q's receive buffer, [world][M / world][N]) at slot `slot`.
int gemm_rs_scatter_bf16(const void* X, const void* W, bool w_mn, void* const* recv, int world, int slot, int M, int N,
                         int K, int* err, int num_sms, cudaStream_t stream) {
  if (world < 1 || world > kMaxTP || M % world || N % 8 || K % 8) return -3;
  if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(W)) & 15) return -4;
  for (int q = 0; q < world; ++q)
    if (reinterpret_cast<uintptr_t>(recv[q]) & 15) return -4;
  CUtensorMap ta, tb;
  if (int rc = make_tmap_bf16_2d(&ta, X, K, M, K, 64, 128)) return -100 - rc;
  if (int rc = w_mn ? make_tmap_bf16_2d(&tb, W, N, K, N, 64, 64) : make_tmap_bf16_2d(&tb, W, K, N, K, 64, 256))
    return -100 - rc;
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.alpha = 1.f; a.err = err;
  a.rs_slot = slot; a.rs_rows = M / world;
  for (int q = 0; q < world; ++q) a.rs_dst[q] = recv[q];
  return w_mn ? launch_gemm<256, false, true, kEpiScatterBF16>(ta, tb, a, num_sms, stream)
              : launch_gemm<256, false, false, kEpiScatterBF16>(ta, tb, a, num_sms, stream);
}

// Operand-ring depth of the CTA-pair kernel for variants 0, 2 and 3.
constexpr int kPairStages = 6;

// Split-K chosen automatically by variant 0: only the tiles of the partial last wave, and only
// for K >= 8192 (128 k-blocks).  Measured on B200 (events, 20 launches, unsplit vs tail split):
// 4096 x 4096 x 14336 0.358 vs 0.341 ms, 4096 x 4096 x 28672 0.706 vs 0.670 ms; at K = 4096 the
// partial tiles' traffic cancels the gain (4096^3 0.104 vs 0.105).  Splitting every tile in two
// (variant 3) lost on every shape (4096^3 0.104 vs 0.134).
constexpr bool kAutoSplit = true;
constexpr int kAutoSplitMinKBlocks = 128;

static bool use_pair_kernel(int M, int N, int variant) {
  return (variant >= 2 && variant <= 6) || (variant == 0 && M >= 512 && N >= 256);
}

// Split plan of the CTA-pair kernel: returns the shares per split tile (1 = no split) and sets
// `*full` to the number of leading tiles that run whole.  The automatic plan (variant 0 when
// kAutoSplit, and variant 6) splits only the tiles of the partial last wave: with `tail` tiles
// left after the full waves of the SM pairs, each is split into s = pairs / tail shares (at most
// 4), so the last round takes 1 / s of a tile instead of a whole one; it is used when that saves
// at least 5 % of the makespan and each share keeps >= 16 k-blocks.  Variant 3 splits every tile
// in two.
int gemm_pair_splits(int M, int N, int K, int variant, int num_sms, int* full) {
  const long long tiles = static_cast<long long>((M + 255) / 256) * ((N + 255) / 256);
  *full = static_cast<int>(tiles);
  if (!use_pair_kernel(M, N, variant) || variant == 2 || variant == 4 || variant == 5) return 1;
  const int kblocks = (K + 63) / 64;
  if (variant == 3) {
    *full = 0;
    return kblocks >= 2 ? 2 : 1;
  }
  if (variant == 0 && !kAutoSplit) return 1;
  const long long pairs = num_sms / 2;
  if (pairs <= 0 || kblocks < (variant == 0 ? kAutoSplitMinKBlocks : 32)) return 1;
  const long long f = tiles / pairs * pairs, tail = tiles - f;
  if (f == 0 || tail == 0) return 1;
  const int shares = static_cast<int>(std::min<long long>({4, pairs / tail, kblocks / 16}));
  if (shares < 2) return 1;
  const double gain = (1.0 - 1.0 / shares) / (static_cast<double>(f / pairs) + 1.0);
  if (gain < 0.05) return 1;
  *full = static_cast<int>(f);
  return shares;
}

// Workspace of a split launch: one 32 x 256 fp32 slot per (split tile, CTA, epilogue warp, share),
// then one counter per (split tile, CTA, epilogue warp).
long long gemm_split_ws_bytes(int M, int N, int splits, int full) {
  const long long tiles = static_cast<long long>((M + 255) / 256) * ((N + 255) / 256);
  const long long tail = tiles - full;
  return tail * 8 * splits * (32LL * 256 * 4) + tail * 8 * 4;
}

// A(m,k) = a_mn ? A[k*lda + m] : A[m*lda + k];  B(n,k) = b_mn ? B[k*ldb + n] : B[n*ldb + k].
// Returns 0 on success, a negative value for a bad argument, else a CUDA error code.
// `split_ws` (gemm_split_ws_bytes(M, N, splits, split_full) bytes, 16-byte aligned) is needed when
// `splits` (gemm_pair_splits) is above 1.
int gemm_bf16(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn,
              void* D, long long ldd, const void* R, long long ldr, int M, int N, int K, int epi,
              float alpha, int* err, int num_sms, cudaStream_t stream, int variant, void* split_ws, int splits,
              int split_full) {
  if (M <= 0 || N <= 0 || K <= 0) return -3;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return -4;
  if ((lda * 2) % 16 || (ldb * 2) % 16) return -5;
  const int esz = (epi == kEpiF32 || epi == kEpiF32Acc) ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(D) & 15) || (ldd * esz) % 16) return -6;
  if (epi == kEpiBF16Res && ((reinterpret_cast<uintptr_t>(R) & 15) || (ldr * 2) % 16)) return -7;
  const int BN = (N <= 128) ? 128 : 256;
  CUtensorMap ta, tb;
  int rc;
  // variant: 0 auto (CTA pair for large tiles, split-K where it fills the last wave), 1 single
  // CTA, 2 CTA pair without split, 3 CTA pair with every tile split in two, 4 CTA pair with a
  // 7-stage ring, 5 CTA pair with 256 x 128 tiles, 6 CTA pair with the partial last wave split
  const bool use_pair = use_pair_kernel(M, N, variant);
  const int stages = variant == 4 ? 7 : kPairStages;
  const int pair_bn = variant == 5 ? 128 : 256;
  if (use_pair) {
    if (!a_mn) rc = make_tmap_bf16_2d(&ta, A, K, M, lda, 64, 128);
    else rc = make_tmap_bf16_2d(&ta, A, M, K, lda, 64, 64);
    if (rc) return -100 - rc;
    if (!b_mn) rc = make_tmap_bf16_2d(&tb, B, K, N, ldb, 64, pair_bn / 2);
    else rc = make_tmap_bf16_2d(&tb, B, N, K, ldb, 64, 64);
    if (rc) return -100 - rc;
    GemmArgs ga{M, N, K, D, ldd, reinterpret_cast<const __nv_bfloat16*>(R), ldr, alpha, err};
    ga.splits = 1;
    if (splits > 1) {
      if (split_ws == nullptr || (reinterpret_cast<uintptr_t>(split_ws) & 15)) return -8;
      const long long tiles = static_cast<long long>((M + 255) / 256) * ((N + 255) / 256);
      if (split_full < 0 || split_full >= tiles || splits > 4) return -9;
      const long long tail = tiles - split_full;
      ga.splits = splits;
      ga.split_full = split_full;
      ga.split_ws = reinterpret_cast<float*>(split_ws);
      ga.split_cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(split_ws) + tail * 8 * splits * (32LL * 256 * 4));
      const cudaError_t e = cudaMemsetAsync(ga.split_cnt, 0, static_cast<size_t>(tail * 8 * 4), stream);
      if (e != cudaSuccess) return static_cast<int>(e);
    }
    switch (epi) {
      case kEpiBF16: return dispatch_major_pair<kEpiBF16>(a_mn, b_mn, ta, tb, ga, num_sms, stream, stages, pair_bn);
      case kEpiF32: return dispatch_major_pair<kEpiF32>(a_mn, b_mn, ta, tb, ga, num_sms, stream, stages, pair_bn);
      case kEpiF32Acc: return dispatch_major_pair<kEpiF32Acc>(a_mn, b_mn, ta, tb, ga, num_sms, stream, stages, pair_bn);
      case kEpiBF16Res: return dispatch_major_pair<kEpiBF16Res>(a_mn, b_mn, ta, tb, ga, num_sms, stream, stages, pair_bn);
    }
    return -2;
  }
  if (!a_mn) rc = make_tmap_bf16_2d(&ta, A, K, M, lda, 64, 128);
  else rc = make_tmap_bf16_2d(&ta, A, M, K, lda, 64, 64);
  if (rc) return -100 - rc;
  if (!b_mn) rc = make_tmap_bf16_2d(&tb, B, K, N, ldb, 64, BN);
  else rc = make_tmap_bf16_2d(&tb, B, N, K, ldb, 64, 64);
  if (rc) return -100 - rc;
  GemmArgs a{M, N, K, D, ldd, reinterpret_cast<const __nv_bfloat16*>(R), ldr, alpha, err};
  if (BN == 128) return dispatch_epi<128>(epi, a_mn, b_mn, ta, tb, a, num_sms, stream);
  return dispatch_epi<256>(epi, a_mn, b_mn, ta, tb, a, num_sms, stream);
}

}  // namespace rb
