// Block-scaled fp8 (E4M3 / E5M2) quantisation and GEMM on the 5th-generation tensor cores.
//
// Quantisation (fp8_quantize_kernel).  A bf16 [R, C] tensor is cut into 128 x 128 tiles, one
// CTA per tile.  Each 1 x 128 block -- a row segment along C ("rowwise") or a column segment
// along R ("colwise") -- or, for weights, each whole 128 x 128 tile ("2-D") gets a power-of-two
// scale s = 2^e, the smallest with amax / s <= the format's largest finite value, and its
// values are stored as fp8(x / s), rounded to nearest even (x / s itself is exact).  The
// colwise output is written transposed ([C, R]) so that every GEMM operand is K-major.  Scales
// are stored K-block major: the scale of operand row r in K-block kb sits at
// kb * kb_stride + (r >> shift) * row_stride: K-block major by default, so a tile's scales for
// one K-block are contiguous, or (rowwise, on request) row major, so that a row's scales travel
// with it when the rows are gathered from other ranks.  Each CTA folds the magnitude of its tile into one atomicMax on the tensor's amax
// word (bit pattern of |x|, so NaN and inf win), the input of the delayed-scaling history.
//
// GEMM.  D[m, n] = alpha * sum_kb sa(m, kb) sb(n, kb) sum_{k in kb} A(m, k) B(n, k) for A [M, K]
// and B [N, K], both K-major fp8, K-blocks of 128.  Two kernels compute it: gemm_fp8_mx_sm100
// (the default, described where it is defined) lets the tensor core apply the scales through
// the block-scaled MMA; gemm_fp8_sm100 (variant 1) promotes each K-block's partial product in
// registers.  The latter, one persistent CTA per SM:
//   warp 0     : TMA producer, 6-deep ring of 128 x 128-byte A and B tiles, 128B swizzle
//   warp 1     : TMEM allocator and single-thread issuer: per K-block four
//                tcgen05.mma.kind::f8f6f4 (K = 32 each) into one of four 128-column TMEM
//                partial accumulators
//   warps 2..9 : promotion and epilogue, two warps per TMEM lane quadrant, each owning 64 of
//                the tile's 128 columns: tcgen05.ld of each finished partial, scaled by
//                sa(row) * sb(column) and added into fp32 registers, then the partial is
//                released -- the MMAs of later K-blocks overlap the scaling of this one.  After
//                the last K-block the same warps store the tile: bf16 (optionally plus a
//                residual), fp32, fp32 accumulate, or bf16 rows scattered to the receive slots of
//                their owner ranks (peer stores over NVLink: the GEMM -> reduce-scatter of a
//                row-parallel layer).
// Power-of-two scales make every scaling exact; the only roundings are the fp8 casts and the
// fp32 accumulation, so a PyTorch emulation reproduces the quantised bytes bit for bit.
//
// New work: the reference framework's fp8 is Transformer Engine inside Megatron-Core
// (`resihp/runtime/generation_hooks.py:83-112` only re-initialises TE buffers) and its
// semantics oracle emulates delayed scaling in float64 (`resihp/runtime/reference_model.py:44-46,
// 204-227`).
#include <cuda.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "act_common.cuh"
#include "fp8_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace rb {
namespace {

enum : int { kF8EpiBF16 = 0, kF8EpiF32 = 1, kF8EpiF32Acc = 2, kF8EpiBF16Res = 3, kF8EpiScatter = 4 };
// Products (2 M N K) below this run the register-promotion kernel by default (see gemm_fp8).
constexpr double kF8SmallFlops = 3.0e10;
constexpr int kF8MaxTP = 8;


// |x| of a bf16 as the bit pattern of an fp32 (an unsigned compare orders magnitudes).
__device__ __forceinline__ uint32_t abs_bits_bf16(uint16_t h) { return static_cast<uint32_t>(h & 0x7fffu) << 16; }

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}


__device__ __forceinline__ float bf16_bits_to_float(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// ------------------------------------------------------------------------------ quantisation
struct QuantArgs {
  const uint16_t* x;  // bf16 bits
  long long ldx;
  int R, C, fmt, two_d;
  int act;  // what is quantised: 0 x itself, 1 gelu(x), 2 silu(x[:, :C]) * x[:, C:] (bf16-rounded)
  int s_row_major;  // 1x128 rowwise scales stored [R][C/128] (a row's scales contiguous) instead of [C/128][R]
  uint8_t* q_row;   // [R, C] or null
  float* s_row;     // 1x128: [C/128][R] (or [R][C/128]);  2-D: [C/128][R/128] (shared by both outputs)
  uint8_t* q_col;  // [C, R] (transposed) or null
  float* s_col;    // 1x128: [R/128][C]
  unsigned int* amax;
};

constexpr int kQT = 128;
constexpr int kQPitch = 136;  // bf16 per shared-memory row (272 bytes: 16-byte aligned, staggered banks)

__global__ void __launch_bounds__(256) fp8_quantize_kernel(QuantArgs p) {
  __shared__ __align__(16) uint16_t tile[kQT * kQPitch];
  __shared__ uint32_t rowmax[kQT];
  __shared__ uint32_t colmax[2][kQT];
  __shared__ uint32_t tile_max;
  const int cb = blockIdx.x, rb = blockIdx.y;
  const int r0 = rb * kQT, c0 = cb * kQT;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int F = fp8_max_exp(p.fmt);

  const int rows = min(kQT, p.R - r0);  // a partial last row tile only in rowwise-only mode
  for (int i = t; i < kQT * 16; i += 256) {
    const int r = i >> 4, c8 = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows) {
      const uint16_t* xr = p.x + static_cast<long long>(r0 + r) * p.ldx + c0 + c8 * 8;
      v = *reinterpret_cast<const uint4*>(xr);
      if (p.act != 0) {  // the activation, rounded to bf16 as the bf16 activation kernels round it
        const uint4 up = p.act == 2 ? *reinterpret_cast<const uint4*>(xr + p.C) : v;
        const uint32_t* a = &v.x;
        const uint32_t* b = &up.x;
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float lo = bf16_bits_to_float(a[k] & 0xffffu), hi = bf16_bits_to_float(a[k] >> 16);
          if (p.act == 1) {
            lo = gelu_tanh(lo);
            hi = gelu_tanh(hi);
          } else {
            lo = silu(lo) * bf16_bits_to_float(b[k] & 0xffffu);
            hi = silu(hi) * bf16_bits_to_float(b[k] >> 16);
          }
          o[k] = pack_bf16x2(lo, hi);
        }
        v = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    *reinterpret_cast<uint4*>(tile + r * kQPitch + c8 * 8) = v;
  }
  __syncthreads();

#pragma unroll 4
  for (int rr = 0; rr < 16; ++rr) {
    const int r = warp * 16 + rr;
    const uint2 u = *reinterpret_cast<const uint2*>(tile + r * kQPitch + lane * 4);
    uint32_t m = max(max(abs_bits_bf16(u.x & 0xffffu), abs_bits_bf16(u.x >> 16)),
                     max(abs_bits_bf16(u.y & 0xffffu), abs_bits_bf16(u.y >> 16)));
    m = warp_max_u32(m);
    if (lane == 0) rowmax[r] = m;
  }
  {
    const int c = t & 127, h = t >> 7;
    uint32_t m = 0;
#pragma unroll 8
    for (int r = h * 64; r < h * 64 + 64; ++r) m = max(m, abs_bits_bf16(tile[r * kQPitch + c]));
    colmax[h][c] = m;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t m = max(max(rowmax[lane], rowmax[lane + 32]), max(rowmax[lane + 64], rowmax[lane + 96]));
    m = warp_max_u32(m);
    if (lane == 0) {
      tile_max = m;
      if (p.amax != nullptr) atomicMax(p.amax, m);
    }
  }
  __syncthreads();
  const uint32_t tmax = tile_max;

  if (p.q_row != nullptr) {
#pragma unroll 4
    for (int rr = 0; rr < 16; ++rr) {
      const int r = warp * 16 + rr;
      if (r >= rows) break;  // uniform across the warp (one row per warp iteration)
      const int e = fp8_scale_exp(p.two_d ? tmax : rowmax[r], F);
      const float inv = exp2_int(-e);
      const uint2 u = *reinterpret_cast<const uint2*>(tile + r * kQPitch + lane * 4);
      const uint32_t q = cvt4_fp8(bf16_bits_to_float(u.x & 0xffffu) * inv, bf16_bits_to_float(u.x >> 16) * inv,
                                  bf16_bits_to_float(u.y & 0xffffu) * inv, bf16_bits_to_float(u.y >> 16) * inv, p.fmt);
      *reinterpret_cast<uint32_t*>(p.q_row + static_cast<long long>(r0 + r) * p.C + c0 + lane * 4) = q;
      if (!p.two_d && lane == 0) {
        const long long si = p.s_row_major ? static_cast<long long>(r0 + r) * (p.C / kQT) + cb
                                           : static_cast<long long>(cb) * p.R + r0 + r;
        p.s_row[si] = exp2_int(e);
      }
    }
  }
  if (p.q_col != nullptr) {
    const int c = t & 127, h = t >> 7;
    const int e = fp8_scale_exp(p.two_d ? tmax : max(colmax[0][c], colmax[1][c]), F);
    const float inv = exp2_int(-e);
    uint8_t* dst = p.q_col + static_cast<long long>(c0 + c) * p.R + r0 + h * 64;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = h * 64 + j * 16 + i * 4;
        w[i] = cvt4_fp8(bf16_bits_to_float(tile[r * kQPitch + c]) * inv,
                        bf16_bits_to_float(tile[(r + 1) * kQPitch + c]) * inv,
                        bf16_bits_to_float(tile[(r + 2) * kQPitch + c]) * inv,
                        bf16_bits_to_float(tile[(r + 3) * kQPitch + c]) * inv, p.fmt);
      }
      *reinterpret_cast<uint4*>(dst + j * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (!p.two_d && h == 0) p.s_col[static_cast<long long>(rb) * p.C + c0 + c] = exp2_int(e);
  }
  if (p.two_d && t == 0) p.s_row[static_cast<long long>(cb) * (p.R / kQT) + rb] = exp2_int(fp8_scale_exp(tmax, F));
}

// ------------------------------------------------------------------------------ GEMM
struct F8GemmArgs {
  int M, N, K;
  uint32_t idesc;
  void* D;
  long long ldd;
  float alpha;
  const float* sa;
  long long sa_kb, sa_row;
  int sa_shift;
  const float* sb;
  long long sb_kb, sb_row;
  int sb_shift;
  int* err;
  // kF8EpiBF16Res: D = alpha * acc + R (bf16, leading dimension ldr)
  const __nv_bfloat16* R;
  long long ldr;
  // kF8EpiScatter (GEMM -> reduce-scatter): row m goes, as bf16, to rank q = m / rs_rows, into
  // slot `rs_slot` of its receive buffer ([world][rs_rows][N], possibly another GPU's memory)
  int rs_slot, rs_rows;
  void* rs_dst[kF8MaxTP];
  // gemm_fp8_mx_sm100: E8M0 scale words packed by mx8_pack_scales, [K-block][128-row group][512 B]
  const uint8_t* sfa;
  const uint8_t* sfb;
  int sfb_groups;  // 128-row groups of B after padding N to the 256-row tile
};

struct F8Cfg {
  static constexpr int BM = 128, BN = 128, BK = 128;  // BK fp8 = 128 bytes = one swizzle row
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr int PARTS = 4;  // TMEM partial accumulators of BN columns
  static constexpr int TMEM_COLS = PARTS * BN;
  static constexpr int NUM_BARS = 2 * STAGES + 2 * PARTS + 1;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 320;
  static constexpr int PROMO_WARPS = 8;
  static constexpr int GROUP_M = 16;
};

// Instruction descriptor of kind::f8f6f4 (f32 accumulation, both operands K-major).
__host__ __device__ constexpr uint32_t make_idesc_f8(int M, int N, int a_fmt, int b_fmt) {
  return (1u << 4) | (static_cast<uint32_t>(a_fmt) << 7) | (static_cast<uint32_t>(b_fmt) << 10) |
         ((static_cast<uint32_t>(N) >> 3) << 17) | ((static_cast<uint32_t>(M) >> 4) << 24);
}

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp gets lane (base + t).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void f8_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = F8Cfg::GROUP_M * num_n;
  const int g = tile / per_group;
  const int first_m = g * F8Cfg::GROUP_M;
  const int gsize = min(num_m - first_m, F8Cfg::GROUP_M);
  const int r = tile - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

__device__ __forceinline__ bool f8_warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int EPI>
__device__ __forceinline__ void f8_store_row(const float (&acc)[64], int row, int col0, const F8GemmArgs& p) {
  if (EPI == kF8EpiBF16 || EPI == kF8EpiBF16Res || EPI == kF8EpiScatter) {
    __nv_bfloat16* dst;
    if (EPI == kF8EpiScatter) {
      const int q = row / p.rs_rows;
      dst = reinterpret_cast<__nv_bfloat16*>(p.rs_dst[q]) +
            (static_cast<long long>(p.rs_slot) * p.rs_rows + (row - q * p.rs_rows)) * p.N + col0;
    } else {
      dst = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd + col0;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = acc[8 * j + i] * p.alpha;
      if (EPI == kF8EpiBF16Res) {
        const uint4 r = *reinterpret_cast<const uint4*>(p.R + row * p.ldr + col0 + 8 * j);
        const float2 f0 = unpack_bf16x2(r.x), f1 = unpack_bf16x2(r.y), f2 = unpack_bf16x2(r.z), f3 = unpack_bf16x2(r.w);
        v[0] += f0.x; v[1] += f0.y; v[2] += f1.x; v[3] += f1.y; v[4] += f2.x; v[5] += f2.y; v[6] += f3.x; v[7] += f3.y;
      }
      uint4 u;
      u.x = pack_bf16x2(v[0], v[1]);
      u.y = pack_bf16x2(v[2], v[3]);
      u.z = pack_bf16x2(v[4], v[5]);
      u.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4*>(dst + 8 * j) = u;
    }
  } else {
    float* dst = reinterpret_cast<float*>(p.D) + row * p.ldd + col0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float4 o = make_float4(acc[4 * j] * p.alpha, acc[4 * j + 1] * p.alpha, acc[4 * j + 2] * p.alpha,
                             acc[4 * j + 3] * p.alpha);
      if (EPI == kF8EpiF32Acc) {
        const float4 old = *reinterpret_cast<const float4*>(dst + 4 * j);
        o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
      }
      *reinterpret_cast<float4*>(dst + 4 * j) = o;
    }
  }
}

// SB_VEC: B's scale differs per output column (1x128 blocks along K for every row of B, laid out
// contiguously over rows); otherwise it is one value per 128-column tile (128 x 128 blocks).
template <bool SB_VEC, int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_fp8_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, F8GemmArgs p) {
  using C = F8Cfg;
  constexpr int STAGES = C::STAGES, PARTS = C::PARTS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * C::B_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto pfull_bar = [&](int j) { return smem_u32(&bars[2 * STAGES + j]); };
  auto pempty_bar = [&](int j) { return smem_u32(&bars[2 * STAGES + PARTS + j]); };
  const uint32_t final_bar = smem_u32(&bars[2 * STAGES + 2 * PARTS]);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int j = 0; j < PARTS; ++j) {
      mbar_init(pfull_bar(j), 1);
      mbar_init(pempty_bar(j), C::PROMO_WARPS);
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

  const int num_m = p.M / C::BM;
  const int num_n = p.N / C::BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = p.K / C::BK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        f8_tile_coords(tile, num_m, num_n, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
          tma_load_2d(smem_u32(sA + stage * C::A_BYTES), &tmA, fb, kb * C::BK, mb * C::BM);
          tma_load_2d(smem_u32(sB + stage * C::B_BYTES), &tmB, fb, kb * C::BK, nb * C::BN);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_parity >> s) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, part = 0;
      uint32_t phase = 0, pphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(pempty_bar(part), pphase ^ 1, abort_flag, p.err) ||
              !mbar_wait(full_bar(stage), phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
          const uint32_t d_tmem = tmem_base + part * C::BN;
#pragma unroll
          for (int k = 0; k < C::BK / 32; ++k) {
            const uint64_t ad = make_smem_desc(a_base + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = make_smem_desc(b_base + k * 32, 16, 1024, kSwizzle128B);
            umma_f8(d_tmem, ad, bd, p.idesc, k != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          umma_commit(pfull_bar(part));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (++part == PARTS) {
            part = 0;
            pphase ^= 1;
          }
        }
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ promotion + epilogue (warps 2..9)
    const int q = warp & 3;             // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;   // which 64 of the tile's 128 columns
    int part = 0;
    uint32_t pphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      f8_tile_coords(tile, num_m, num_n, mb, nb);
      const int row = mb * C::BM + q * 32 + lane;
      const int col0 = nb * C::BN + half * 64;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      bool ok = true;
#pragma unroll 1
      for (int kb = 0; kb < kblocks; ++kb) {
        const float sa = __ldg(p.sa + kb * p.sa_kb + static_cast<long long>(row >> p.sa_shift) * p.sa_row);
        float s_tile = 0.f;
        if (!SB_VEC) s_tile = sa * __ldg(p.sb + kb * p.sb_kb + static_cast<long long>(col0 >> p.sb_shift) * p.sb_row);
        if (!f8_warp_wait(pfull_bar(part), pphase, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + part * C::BN + half * 64;
        if (SB_VEC) {
          // 16 columns at a time: per-column scales cost 4 more registers per column group
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(tbase + c * 16, r);
            const float4* sbp = reinterpret_cast<const float4*>(p.sb + kb * p.sb_kb + col0 + c * 16);
            float4 sv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) sv[i] = __ldg(sbp + i);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              acc[c * 16 + 4 * i + 0] = fmaf(__uint_as_float(r[4 * i + 0]), sa * sv[i].x, acc[c * 16 + 4 * i + 0]);
              acc[c * 16 + 4 * i + 1] = fmaf(__uint_as_float(r[4 * i + 1]), sa * sv[i].y, acc[c * 16 + 4 * i + 1]);
              acc[c * 16 + 4 * i + 2] = fmaf(__uint_as_float(r[4 * i + 2]), sa * sv[i].z, acc[c * 16 + 4 * i + 2]);
              acc[c * 16 + 4 * i + 3] = fmaf(__uint_as_float(r[4 * i + 3]), sa * sv[i].w, acc[c * 16 + 4 * i + 3]);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[c * 32 + j] = fmaf(__uint_as_float(r[j]), s_tile, acc[c * 32 + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pempty_bar(part));
        if (++part == PARTS) {
          part = 0;
          pphase ^= 1;
        }
      }
      if (!ok) break;
      f8_store_row<EPI>(acc, row, col0, p);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <bool SB_VEC, int EPI>
int launch_fp8(const CUtensorMap& ta, const CUtensorMap& tb, const F8GemmArgs& a, int num_sms, cudaStream_t s) {
  auto kern = gemm_fp8_sm100<SB_VEC, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, F8Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  const int tiles = (a.M / F8Cfg::BM) * (a.N / F8Cfg::BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  kern<<<grid, F8Cfg::THREADS, F8Cfg::SMEM_BYTES, s>>>(ta, tb, a);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------- hardware block-scaled GEMM
// gemm_fp8_mx_sm100: the same product with the scales applied by the tensor core
// (tcgen05.mma.kind::mxf8f6f4.block_scale, one E8M0 scale per 32 K-elements of every A row and
// every B row).  A power-of-two 1 x 128 (or 128 x 128) scale 2^e is the E8M0 byte e + 127,
// repeated over the four 32-deep sub-blocks of its 128-deep K-block, so the hardware applies
// exactly the scales the promotion kernel applies, and no promotion warps or partial
// accumulators are needed.  Per CTA: a 128 x 256 output tile, 4-deep ring of 128 x 128-byte A and
// 256 x 128-byte B tiles plus the K-block's scale factors, single 256-column TMEM accumulator.
//   warp 0     : producer (one thread): per K-block the A and B tiles by TMA and the K-block's
//                scale words by two untiled bulk copies, all on one barrier.  The words are
//                packed beforehand by mx8_pack_scales in the layout tcgen05.cp expects (row r of
//                a 128-row group: 16-byte row r % 32, word r / 32, the E8M0 byte four times), so
//                the scales travel like the operands: no register round trip, no proxy fence.
//   warp 1     : TMEM allocator and single-thread issuer: per K-block three tcgen05.cp
//                (32x128b.warpx4: A's 128 rows into 4 columns, B's 256 rows into 8 columns,
//                two alternating column sets) and four block-scaled MMAs (K = 32 each).
//   warps 2..9 : epilogue, two warps per TMEM lane quadrant, 128 columns each: the whole row
//                segment is read into registers, the accumulator is released at once (the next
//                tile's MMAs start while these warps convert and store), then stored.
struct Mx8Cfg {
  static constexpr int BM = 128, BN = 256, BK = 128;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int SFA_BYTES = 512;            // 128 rows x one 32-bit word of E8M0 bytes
  static constexpr int SF_BYTES = SFA_BYTES * 3;   // A, then B's two 128-row groups
  static constexpr int STAGES = 4;
  static constexpr int TMEM_COLS = 512;  // accumulator in 0..255, scale factors from column 256
  static constexpr int SF_COL = 256;
  static constexpr int NUM_BARS = 2 * STAGES + 3;
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES + SF_BYTES) + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 320;
  static constexpr int EPI_WARPS = 8;
  static constexpr int GROUP_M = 16;
  static_assert(SMEM_BYTES <= 232448, "over the 227 KB of dynamic shared memory a CTA may have");
};

// Instruction descriptor of kind::mxf8f6f4.block_scale: A / B formats (E4M3 0, E5M2 1), K-major
// operands, N >> 3 at bit 17, E8M0 scale factors (bit 23), M >> 4 at bit 24; the scale-factor
// byte selectors (bits 4-5 for B, 29-30 for A) stay 0: every byte of a scale word is the same.
__host__ __device__ constexpr uint32_t make_idesc_mx8(int M, int N, int a_fmt, int b_fmt) {
  return (static_cast<uint32_t>(a_fmt) << 7) | (static_cast<uint32_t>(b_fmt) << 10) |
         ((static_cast<uint32_t>(N) >> 3) << 17) | (1u << 23) | ((static_cast<uint32_t>(M) >> 4) << 24);
}

__device__ __forceinline__ void umma_mx8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Shared memory -> TMEM copy of 32 rows x 16 bytes, broadcast to all four 32-lane quadrants:
// TMEM lane 32 q + l, columns 0..3, get bytes 16 l .. 16 l + 15 of the block.
__device__ __forceinline__ void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// E8M0 byte of a power-of-two fp32 scale, repeated in all four bytes of a word.
__device__ __forceinline__ uint32_t e8m0_word(float s) { return ((__float_as_uint(s) >> 23) & 0xffu) * 0x01010101u; }

// Packs fp32 power-of-two scales (scale of row r in K-block kb at s[kb * s_kb + (r >> shift) *
// s_row]) into E8M0 words for the block-scaled GEMM: for K-block kb and 128-row group g, a
// 512-byte block at (kb * groups + g) * 512 whose word (r % 32) * 4 + (r % 128) / 32 holds row r's
// byte four times.  Rows in [rows, rows_pad) get scale 1 (their operand rows are zero-filled).
__global__ void mx8_pack_scales(const float* __restrict__ s, long long s_kb, long long s_row, int shift, int rows,
                                int rows_pad, int kblocks, uint32_t* __restrict__ out) {
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= static_cast<long long>(rows_pad) * kblocks) return;
  const int kb = static_cast<int>(t / rows_pad), r = static_cast<int>(t % rows_pad);
  const int rr = r & 127;
  const uint32_t w = r < rows ? e8m0_word(s[kb * s_kb + static_cast<long long>(r >> shift) * s_row]) : 0x7f7f7f7fu;
  out[(static_cast<long long>(kb) * (rows_pad / 128) + (r >> 7)) * 128 + (rr & 31) * 4 + (rr >> 5)] = w;
}

__device__ __forceinline__ void mx8_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = Mx8Cfg::GROUP_M * num_n;
  const int g = tile / per_group;
  const int first_m = g * Mx8Cfg::GROUP_M;
  const int gsize = min(num_m - first_m, Mx8Cfg::GROUP_M);
  const int r = tile - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

template <int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_fp8_mx_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      F8GemmArgs p) {
  using C = Mx8Cfg;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* sSF = sB + STAGES * C::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSF + STAGES * C::SF_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  const uint32_t tfull_bar = smem_u32(&bars[2 * STAGES]);
  const uint32_t tempty_bar = smem_u32(&bars[2 * STAGES + 1]);
  const uint32_t final_bar = smem_u32(&bars[2 * STAGES + 2]);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, C::EPI_WARPS);
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

  const int num_m = p.M / C::BM;
  const int num_n = (p.N + C::BN - 1) / C::BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = p.K / C::BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      const int a_groups = p.M / 128;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        mx8_tile_coords(tile, num_m, num_n, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::A_BYTES + C::B_BYTES + C::SF_BYTES);
          tma_load_2d(smem_u32(sA + stage * C::A_BYTES), &tmA, fb, kb * C::BK, mb * C::BM);
          tma_load_2d(smem_u32(sB + stage * C::B_BYTES), &tmB, fb, kb * C::BK, nb * C::BN);
          const uint32_t sf = smem_u32(sSF + stage * C::SF_BYTES);
          bulk_load_1d(sf, p.sfa + (static_cast<long long>(kb) * a_groups + mb) * C::SFA_BYTES, C::SFA_BYTES, fb);
          bulk_load_1d(sf + C::SFA_BYTES, p.sfb + (static_cast<long long>(kb) * p.sfb_groups + 2 * nb) * C::SFA_BYTES,
                       2 * C::SFA_BYTES, fb);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_parity >> s) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, set = 0;
      uint32_t phase = 0, tphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(tempty_bar, tphase ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf = smem_u32(sSF + stage * C::SF_BYTES);
          const uint32_t t_sfa = tmem_base + C::SF_COL + set * 16;
          const uint32_t t_sfb = t_sfa + 4;
          // 32 rows of 16 bytes: 8-row core matrices 128 bytes apart, no swizzle
          tmem_cp_32x128b_warpx4(t_sfa, make_smem_desc(sf, 128, 128, kSwizzleNone));
          tmem_cp_32x128b_warpx4(t_sfb, make_smem_desc(sf + C::SFA_BYTES, 128, 128, kSwizzleNone));
          tmem_cp_32x128b_warpx4(t_sfb + 4, make_smem_desc(sf + 2 * C::SFA_BYTES, 128, 128, kSwizzleNone));
          const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 32; ++k) {
            const uint64_t ad = make_smem_desc(a_base + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = make_smem_desc(b_base + k * 32, 16, 1024, kSwizzle128B);
            umma_mx8(tmem_base, ad, bd, p.idesc, t_sfa, t_sfb, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          set ^= 1;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar);
        tphase ^= 1;
      }
      umma_commit(final_bar);
      mbar_wait(final_bar, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint32_t tphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      mx8_tile_coords(tile, num_m, num_n, mb, nb);
      if (!f8_warp_wait(tfull_bar, tphase, abort_flag, p.err)) break;
      tphase ^= 1;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + half * 128;
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld_32x32b_x32(tb, r0);
      tmem_ld_32x32b_x32(tb + 32, r1);
      tmem_ld_32x32b_x32(tb + 64, r2);
      tmem_ld_32x32b_x32(tb + 96, r3);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar);  // the next tile's MMAs may overwrite the accumulator
      const int row = mb * C::BM + q * 32 + lane;
      const int col0 = nb * C::BN + half * 128;
      if (col0 < p.N) {
        float v[64];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r0[j]);
          v[32 + j] = __uint_as_float(r1[j]);
        }
        f8_store_row<EPI>(v, row, col0, p);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r2[j]);
          v[32 + j] = __uint_as_float(r3[j]);
        }
        f8_store_row<EPI>(v, row, col0 + 64, p);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int EPI>
int launch_mx8(const CUtensorMap& ta, const CUtensorMap& tb, const F8GemmArgs& a, int num_sms, cudaStream_t s) {
  auto kern = gemm_fp8_mx_sm100<EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Mx8Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  const int tiles = (a.M / Mx8Cfg::BM) * ((a.N + Mx8Cfg::BN - 1) / Mx8Cfg::BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  kern<<<grid, Mx8Cfg::THREADS, Mx8Cfg::SMEM_BYTES, s>>>(ta, tb, a);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------- CTA-pair block-scaled GEMM
// gemm_fp8_mx_pair_sm100: the block-scaled product on a CTA pair (cta_group::2), 256 x 256
// output tiles.  Each CTA holds its 128 rows of A, its 128 rows of the tile's 256 B rows, the
// scale words of its A rows and those of all 256 B rows (the tensor core of each CTA scales its
// half of D by every column's B scale).  Per CTA and K-block that is 33.5 KB instead of the
// single-CTA kernel's 49.5 KB for the same MMA time, so the 6-stage ring covers twice the load
// latency.  All loads of both CTAs (tiles and scale words, the latter through an unswizzled
// tensor map over the packed words) complete on the leader's stage barrier; the leader's single
// thread issues per K-block three tcgen05.cp.cta_group::2 (each CTA's words into its own TMEM)
// and four MMAs of 256 x 256 x 32, and commits to both CTAs' barriers.  Epilogue as in the
// single-CTA kernel: eight warps per CTA drain their 128-column row segments into registers and
// release the accumulator (16 arrivals on the leader's barrier) before storing.
struct Mx8PairCfg {
  static constexpr int BM = 128;   // rows per CTA (the pair covers 256)
  static constexpr int BN = 256;   // columns of the pair's tile
  static constexpr int BNH = 128;  // B rows held per CTA
  static constexpr int BK = 128;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BNH * BK;
  static constexpr int SFA_BYTES = 512;
  static constexpr int SF_BYTES = 3 * SFA_BYTES;  // this CTA's A rows, then all 256 B rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SF_BYTES;
  static constexpr int STAGES = 6;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SF_COL = 256;
  static constexpr int NUM_BARS = 2 * STAGES + 3;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 320;
  static constexpr int EPI_WARPS = 8;
  static constexpr int GROUP_M = 8;  // in 256-row pair tiles
  static_assert(SMEM_BYTES <= 232448, "over the 227 KB of dynamic shared memory a CTA may have");
};

__device__ __forceinline__ void umma_mx8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

__device__ __forceinline__ void tmem_cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void mx8p_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = Mx8PairCfg::GROUP_M * num_n;
  const int g = tile / per_group;
  const int first_m = g * Mx8PairCfg::GROUP_M;
  const int gsize = min(num_m - first_m, Mx8PairCfg::GROUP_M);
  const int r = tile - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    gemm_fp8_mx_pair_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmS, F8GemmArgs p) {
  using C = Mx8PairCfg;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* sSF = sB + STAGES * C::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSF + STAGES * C::SF_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  const uint32_t tfull_bar = smem_u32(&bars[2 * STAGES]);
  const uint32_t tempty_bar = smem_u32(&bars[2 * STAGES + 1]);
  const uint32_t final_bar = smem_u32(&bars[2 * STAGES + 2]);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const bool leader = cta == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 2 * C::EPI_WARPS);
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmS);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = p.M / (2 * C::BM);
  const int num_n = (p.N + C::BN - 1) / C::BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = p.K / C::BK;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int a_groups = p.M / 128;
  const int sfb_row0 = kblocks * a_groups;  // packed words: A's blocks, then B's

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += num_pairs) {
        int mb, nb;
        mx8p_tile_coords(tile, num_m, num_n, mb, nb);
        const int m0 = mb * 2 * C::BM + static_cast<int>(cta) * C::BM;
        const int n0 = nb * C::BN + static_cast<int>(cta) * C::BNH;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = full_bar(stage);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * C::STAGE_BYTES);
          const uint32_t fb = mapa_shared(fb_local, 0);
          const uint32_t sf = smem_u32(sSF + stage * C::SF_BYTES);
          tma_load_2d_pair(smem_u32(sA + stage * C::A_BYTES), &tmA, fb, kb * C::BK, m0);
          tma_load_2d_pair(smem_u32(sB + stage * C::B_BYTES), &tmB, fb, kb * C::BK, n0);
          tma_load_2d_pair(sf, &tmS, fb, 0, kb * a_groups + 2 * mb + static_cast<int>(cta));
          tma_load_2d_pair(sf + C::SFA_BYTES, &tmS, fb, 0, sfb_row0 + kb * p.sfb_groups + 2 * nb);
          tma_load_2d_pair(sf + 2 * C::SFA_BYTES, &tmS, fb, 0, sfb_row0 + kb * p.sfb_groups + 2 * nb + 1);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // the leader's barriers count both CTAs' loads; the peer's loads of a stage complete
      // before the leader's barrier phase does
      if (leader)
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(full_bar(s), (issued_parity >> s) & 1, nullptr, p.err, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      int stage = 0, set = 0;
      uint32_t phase = 0, tphase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        if (!mbar_wait(tempty_bar, tphase ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf = smem_u32(sSF + stage * C::SF_BYTES);
          const uint32_t t_sfa = tmem_base + C::SF_COL + set * 16;
          const uint32_t t_sfb = t_sfa + 4;
          tmem_cp_32x128b_warpx4_pair(t_sfa, make_smem_desc(sf, 128, 128, kSwizzleNone));
          tmem_cp_32x128b_warpx4_pair(t_sfb, make_smem_desc(sf + C::SFA_BYTES, 128, 128, kSwizzleNone));
          tmem_cp_32x128b_warpx4_pair(t_sfb + 4, make_smem_desc(sf + 2 * C::SFA_BYTES, 128, 128, kSwizzleNone));
          const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 32; ++k) {
            const uint64_t ad = make_smem_desc(a_base + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = make_smem_desc(b_base + k * 32, 16, 1024, kSwizzle128B);
            umma_mx8_pair(tmem_base, ad, bd, p.idesc, t_sfa, t_sfb, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(empty_bar(stage));
          umma_commit_pair(mapa_shared(empty_bar(stage), 1));
          set ^= 1;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar);
        umma_commit_pair(mapa_shared(tfull_bar, 1));
        tphase ^= 1;
      }
      umma_commit_pair(final_bar);
      mbar_wait(final_bar, 0, nullptr, p.err, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t release = leader ? tempty_bar : mapa_shared(tempty_bar, 0);
    uint32_t tphase = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs) {
      int mb, nb;
      mx8p_tile_coords(tile, num_m, num_n, mb, nb);
      if (!f8_warp_wait(tfull_bar, tphase, abort_flag, p.err)) break;
      tphase ^= 1;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + half * 128;
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld_32x32b_x32(tb, r0);
      tmem_ld_32x32b_x32(tb + 32, r1);
      tmem_ld_32x32b_x32(tb + 64, r2);
      tmem_ld_32x32b_x32(tb + 96, r3);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(release);
        else mbar_arrive_cluster(release);
      }
      const int row = mb * 2 * C::BM + static_cast<int>(cta) * C::BM + q * 32 + lane;
      const int col0 = nb * C::BN + half * 128;
      if (col0 < p.N) {
        float v[64];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r0[j]);
          v[32 + j] = __uint_as_float(r1[j]);
        }
        f8_store_row<EPI>(v, row, col0, p);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r2[j]);
          v[32 + j] = __uint_as_float(r3[j]);
        }
        f8_store_row<EPI>(v, row, col0 + 64, p);
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs may still read its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

template <int EPI>
int launch_mx8_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ts, const F8GemmArgs& a,
                    int num_sms, cudaStream_t s) {
  auto kern = gemm_fp8_mx_pair_sm100<EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Mx8PairCfg::SMEM_BYTES);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  const int tiles = (a.M / (2 * Mx8PairCfg::BM)) * ((a.N + Mx8PairCfg::BN - 1) / Mx8PairCfg::BN);
  int pairs = num_sms / 2;
  if (tiles < pairs) pairs = tiles;
  kern<<<2 * pairs, Mx8PairCfg::THREADS, Mx8PairCfg::SMEM_BYTES, s>>>(ta, tb, ts, a);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

long long gemm_fp8_sf_bytes(int M, int N, int K) {
  const long long n_pad = (N + Mx8Cfg::BN - 1) / Mx8Cfg::BN * Mx8Cfg::BN;
  return 4LL * (K / 128) * (M + n_pad);
}

int fp8_quantize(const void* x, long long ldx, int R, int C, int fmt, int two_d, void* q_row, float* s_row,
                 void* q_col, float* s_col, unsigned int* amax, cudaStream_t s, int s_row_major, int act) {
  if (R <= 0 || C <= 0 || C % kQT || (fmt != kFp8E4M3 && fmt != kFp8E5M2)) return -3;
  if (R % kQT && (two_d || q_col != nullptr)) return -3;  // 128-row blocks need whole row tiles
  if (act < 0 || act > 2) return -3;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || ldx % 8 || ldx < (act == 2 ? 2 * C : C)) return -4;
  if ((q_row != nullptr && s_row == nullptr) || (q_col != nullptr && !two_d && s_col == nullptr)) return -5;
  if (two_d && s_row == nullptr) return -5;
  if ((q_row != nullptr && (reinterpret_cast<uintptr_t>(q_row) & 15)) ||
      (q_col != nullptr && (reinterpret_cast<uintptr_t>(q_col) & 15)))
    return -6;
  if (s_row_major && two_d) return -3;
  QuantArgs p{static_cast<const uint16_t*>(x), ldx, R, C, fmt, two_d, act, s_row_major, static_cast<uint8_t*>(q_row),
              s_row, static_cast<uint8_t*>(q_col), s_col, amax};
  dim3 grid(C / kQT, (R + kQT - 1) / kQT);
  fp8_quantize_kernel<<<grid, 256, 0, s>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int gemm_fp8(const void* A, int a_fmt, const void* B, int b_fmt, const float* sa, long long sa_kb, long long sa_row,
             int sa_shift, const float* sb, long long sb_kb, long long sb_row, int sb_shift, void* D, long long ldd,
             int M, int N, int K, int epi, float alpha, int* err, int num_sms, cudaStream_t stream, const void* R,
             long long ldr, void* const* rs_dst, int world, int rs_slot, int variant, void* sf_ws) {
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128 || K % 128) return -3;
  if (variant < 0 || variant > 3) return -3;
  if ((a_fmt != kFp8E4M3 && a_fmt != kFp8E5M2) || (b_fmt != kFp8E4M3 && b_fmt != kFp8E5M2)) return -3;
  if ((sa_shift != 0 && sa_shift != 7) || (sb_shift != 0 && sb_shift != 7)) return -3;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return -4;
  F8GemmArgs a{};
  if (epi == kF8EpiScatter) {
    if (world < 1 || world > kF8MaxTP || M % world || rs_slot < 0) return -8;
    for (int q = 0; q < world; ++q) {
      if (rs_dst[q] == nullptr || (reinterpret_cast<uintptr_t>(rs_dst[q]) & 15)) return -8;
      a.rs_dst[q] = rs_dst[q];
    }
    a.rs_slot = rs_slot;
    a.rs_rows = M / world;
  } else {
    const int esz = (epi == kF8EpiBF16 || epi == kF8EpiBF16Res) ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(D) & 15) || (ldd * esz) % 16 || ldd < N) return -6;
  }
  if (epi == kF8EpiBF16Res && (R == nullptr || (reinterpret_cast<uintptr_t>(R) & 15) || ldr % 8 || ldr < N)) return -9;
  const bool sb_vec = sb_shift == 0;
  // variant 2: tensor-core scaling on single CTAs; 1: register promotion; 3: tensor-core scaling
  // on CTA pairs (M a multiple of 256).  Measured at 8192^3 (events, same box): single CTAs
  // 0.464-0.479 ms, CTA pairs 0.493 ms, so the pair is not the default.  Variant 0 (default) is
  // variant 2, except for products under kF8SmallFlops, which take the register-promotion kernel:
  // it needs no scale-packing launches, and on these sizes those cost more than the promotion
  // (4096 x 1024 x 2048: 0.041 / 0.038 ms against 0.045 / 0.042 in two runs; 4096 x 3072 x 2048:
  // 0.081 against 0.063, so the threshold sits between them).
  const bool promotable = !sb_vec || (sb_row == 1 && sb_kb % 4 == 0 && !(reinterpret_cast<uintptr_t>(sb) & 15));
  const bool small = variant == 0 && 2.0 * M * N * K < kF8SmallFlops && promotable;
  const bool mx = variant != 1 && !small;
  const bool pair = variant == 3;
  if (pair && M % 256) return -3;
  if (!mx && sb_vec && (sb_row != 1 || sb_kb % 4 || (reinterpret_cast<uintptr_t>(sb) & 15))) return -7;
  CUtensorMap ta, tb;
  if (int rc = make_tmap_2d_sw128(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, K, M, K, 128, 128)) return -100 - rc;
  const uint32_t b_box = (mx && !pair) ? Mx8Cfg::BN : 128;
  if (int rc = make_tmap_2d_sw128(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, B, K, N, K, 128, b_box)) return -100 - rc;
  a.M = M; a.N = N; a.K = K;
  a.idesc = pair ? make_idesc_mx8(2 * Mx8PairCfg::BM, Mx8PairCfg::BN, a_fmt, b_fmt)
                 : mx ? make_idesc_mx8(Mx8Cfg::BM, Mx8Cfg::BN, a_fmt, b_fmt) : make_idesc_f8(128, 128, a_fmt, b_fmt);
  a.D = D; a.ldd = ldd; a.alpha = alpha;
  a.sa = sa; a.sa_kb = sa_kb; a.sa_row = sa_row; a.sa_shift = sa_shift;
  a.sb = sb; a.sb_kb = sb_kb; a.sb_row = sb_row; a.sb_shift = sb_shift;
  a.err = err;
  a.R = static_cast<const __nv_bfloat16*>(R); a.ldr = ldr;
  if (mx) {
    if (sf_ws == nullptr || (reinterpret_cast<uintptr_t>(sf_ws) & 15)) return -10;
    const int kblocks = K / 128;
    const int n_pad = (N + Mx8Cfg::BN - 1) / Mx8Cfg::BN * Mx8Cfg::BN;
    uint32_t* wa = static_cast<uint32_t*>(sf_ws);
    uint32_t* wb = wa + static_cast<long long>(kblocks) * M;  // one word per row per K-block
    const long long na = static_cast<long long>(kblocks) * M, nb = static_cast<long long>(kblocks) * n_pad;
    mx8_pack_scales<<<static_cast<unsigned>((na + 255) / 256), 256, 0, stream>>>(sa, sa_kb, sa_row, sa_shift, M, M,
                                                                                 kblocks, wa);
    mx8_pack_scales<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, stream>>>(sb, sb_kb, sb_row, sb_shift, N,
                                                                                 n_pad, kblocks, wb);
    a.sfa = reinterpret_cast<const uint8_t*>(wa);
    a.sfb = reinterpret_cast<const uint8_t*>(wb);
    a.sfb_groups = n_pad / 128;
    if (pair) {
      // the packed words as rows of 512 bytes (128 words): A's K-block-major blocks, then B's
      CUtensorMap ts;
      const uint64_t rows = static_cast<uint64_t>(kblocks) * (M + n_pad) / 128;
      if (int rc = make_tmap_2d_plain(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, sf_ws, 128, rows, 128, 128, 1))
        return -100 - rc;
      switch (epi) {
        case kF8EpiBF16: return launch_mx8_pair<kF8EpiBF16>(ta, tb, ts, a, num_sms, stream);
        case kF8EpiF32: return launch_mx8_pair<kF8EpiF32>(ta, tb, ts, a, num_sms, stream);
        case kF8EpiF32Acc: return launch_mx8_pair<kF8EpiF32Acc>(ta, tb, ts, a, num_sms, stream);
        case kF8EpiBF16Res: return launch_mx8_pair<kF8EpiBF16Res>(ta, tb, ts, a, num_sms, stream);
        case kF8EpiScatter: return launch_mx8_pair<kF8EpiScatter>(ta, tb, ts, a, num_sms, stream);
      }
      return -2;
    }
    switch (epi) {
      case kF8EpiBF16: return launch_mx8<kF8EpiBF16>(ta, tb, a, num_sms, stream);
      case kF8EpiF32: return launch_mx8<kF8EpiF32>(ta, tb, a, num_sms, stream);
      case kF8EpiF32Acc: return launch_mx8<kF8EpiF32Acc>(ta, tb, a, num_sms, stream);
      case kF8EpiBF16Res: return launch_mx8<kF8EpiBF16Res>(ta, tb, a, num_sms, stream);
      case kF8EpiScatter: return launch_mx8<kF8EpiScatter>(ta, tb, a, num_sms, stream);
    }
    return -2;
  }
  switch (epi) {
    case kF8EpiBF16: return sb_vec ? launch_fp8<true, kF8EpiBF16>(ta, tb, a, num_sms, stream)
                                   : launch_fp8<false, kF8EpiBF16>(ta, tb, a, num_sms, stream);
    case kF8EpiF32: return sb_vec ? launch_fp8<true, kF8EpiF32>(ta, tb, a, num_sms, stream)
                                  : launch_fp8<false, kF8EpiF32>(ta, tb, a, num_sms, stream);
    case kF8EpiF32Acc: return sb_vec ? launch_fp8<true, kF8EpiF32Acc>(ta, tb, a, num_sms, stream)
                                     : launch_fp8<false, kF8EpiF32Acc>(ta, tb, a, num_sms, stream);
    case kF8EpiBF16Res: return sb_vec ? launch_fp8<true, kF8EpiBF16Res>(ta, tb, a, num_sms, stream)
                                      : launch_fp8<false, kF8EpiBF16Res>(ta, tb, a, num_sms, stream);
    case kF8EpiScatter: return sb_vec ? launch_fp8<true, kF8EpiScatter>(ta, tb, a, num_sms, stream)
                                      : launch_fp8<false, kF8EpiScatter>(ta, tb, a, num_sms, stream);
  }
  return -2;
}

}  // namespace rb
