// Causal multi-head attention with grouped KV heads (GQA), forward and backward, on
// warp-level mma.sync (m16n8k16 bf16 -> f32).  This is the portable path of the package:
// it runs any head count / sequence length, and serves as the numerical cross-check of the
// tcgen05 attention kernel.
//
// Layout: token-major rows (row = b * S + s).  q/k/v/o/dq/dk/dv are strided row views, head h
// at columns [h * D, (h + 1) * D) of its view.  Softmax statistics (lse, delta) are
// [B, Hq, S] fp32.  Backward is deterministic: dK/dV are accumulated by one CTA per KV block
// (looping over the q heads of the group and over q blocks), dQ by one CTA per q block.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "sm100.cuh"

namespace rb {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Tile of ROWS x D bf16 in shared memory; 16-byte chunk c of row r lives at chunk (c ^ (r & 7)).
template <int D>
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int c_elem) {
  const int chunk = c_elem >> 3;
  return base + r * (D * 2) + (((chunk ^ (r & 7))) << 4) + ((c_elem & 7) << 1);
}

// Asynchronously copy rows [r0, r0 + ROWS) of a strided global view into a swizzled tile;
// rows >= S are zero-filled.
template <int ROWS, int D, int THREADS>
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g, long long stride, int r0, int S) {
  constexpr int CH = D / 8;
  for (int i = threadIdx.x; i < ROWS * CH; i += THREADS) {
    const int r = i / CH, c = i % CH;
    const bool ok = (r0 + r) < S;
    const __nv_bfloat16* src = g + (ok ? static_cast<long long>(r0 + r) * stride : 0) + c * 8;
    cp_async16(sbase + r * (D * 2) + ((c ^ (r & 7)) << 4), src, ok);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

// ------------------------------------------------------------------------------------------ forward
// CTA: BM = 16 * WARPS query rows of one (b, h); loops over key blocks of BN rows.
template <int D, int WARPS, int BN>
__global__ void __launch_bounds__(WARPS * 32) attn_fwd_kernel(AttnArgs p) {
  constexpr int BM = 16 * WARPS;
  constexpr int THREADS = WARPS * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BM * D * 2;
  const uint32_t sV0 = sK0 + 2 * BN * D * 2;

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * BM;
  const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(p.q) + static_cast<long long>(b) * p.S * p.q_stride + h * D;
  const __nv_bfloat16* kg = reinterpret_cast<const __nv_bfloat16*>(p.k) + static_cast<long long>(b) * p.S * p.k_stride + hk * D;
  const __nv_bfloat16* vg = reinterpret_cast<const __nv_bfloat16*>(p.v) + static_cast<long long>(b) * p.S * p.v_stride + hk * D;

  const int kv_end = p.causal ? min(p.S, q0 + BM) : p.S;
  const int nkb = (kv_end + BN - 1) / BN;

  load_tile<BM, D, THREADS>(sQ, qg, p.q_stride, q0, p.S);
  cp_commit();
  if (nkb > 0) {
    load_tile<BN, D, THREADS>(sK0, kg, p.k_stride, 0, p.S);
    load_tile<BN, D, THREADS>(sV0, vg, p.v_stride, 0, p.S);
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();

  // Q fragments of this warp's 16 rows, all of D.
  uint32_t qf[D / 16][4];
  {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c = kk * 16 + (lane >> 4) * 8;
      ldsm_x4(swz<D>(sQ, r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = p.scale * kLog2e;
  const int g = lane >> 2, t4 = lane & 3;
  const int row_a = q0 + warp * 16 + g;  // global query rows of this thread
  const int row_b = row_a + 8;

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    const uint32_t sK = sK0 + buf * BN * D * 2, sV = sV0 + buf * BN * D * 2;
    if (j + 1 < nkb) {
      load_tile<BN, D, THREADS>(sK0 + (buf ^ 1) * BN * D * 2, kg, p.k_stride, (j + 1) * BN, p.S);
      load_tile<BN, D, THREADS>(sV0 + (buf ^ 1) * BN * D * 2, vg, p.v_stride, (j + 1) * BN, p.S);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();

    float s[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < BN / 16; ++n2) {
        uint32_t b0, b1, b2, b3;
        const int r = n2 * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(swz<D>(sK, r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * n2], qf[kk], b0, b1);
        mma_bf16(s[2 * n2 + 1], qf[kk], b2, b3);
      }
    }
    const int kbase = j * BN;
    const bool need_mask = (kbase + BN > p.S) || (p.causal && kbase + BN - 1 > q0 + warp * 16);
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = kbase + n * 8 + t4 * 2 + (e & 1);
        const int row = (e < 2) ? row_a : row_b;
        float x = s[n][e];
        if (need_mask && (col >= p.S || (p.causal && col > row))) x = -INFINITY;
        s[n][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float alpha[2], mref[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mref[i] = (mx[i] == -INFINITY) ? 0.f : mx[i] * sl2;
      alpha[i] = (m_r[i] == -INFINITY) ? 0.f : exp2f(m_r[i] * sl2 - mref[i]);
      m_r[i] = mx[i];
      l_r[i] *= alpha[i];
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      const float p0 = exp2f(s[n][0] * sl2 - mref[0]);
      const float p1 = exp2f(s[n][1] * sl2 - mref[0]);
      const float p2 = exp2f(s[n][2] * sl2 - mref[1]);
      const float p3 = exp2f(s[n][3] * sl2 - mref[1]);
      l_r[0] += p0 + p1;
      l_r[1] += p2 + p3;
      pf[n >> 1][(n & 1) * 2 + 0] = pack2(p0, p1);
      pf[n >> 1][(n & 1) * 2 + 1] = pack2(p2, p3);
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int n2 = 0; n2 < D / 16; ++n2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = n2 * 16 + (lane >> 4) * 8;
        ldsm_x4_t(swz<D>(sV, r, c), b0, b1, b2, b3);
        mma_bf16(o[2 * n2], a, b0, b1);
        mma_bf16(o[2 * n2 + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();

#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 1);
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 2);
  }
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  __nv_bfloat16* og = reinterpret_cast<__nv_bfloat16*>(p.o) + static_cast<long long>(b) * p.S * p.o_stride + h * D;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + t4 * 2;
    if (row_a < p.S)
      *reinterpret_cast<uint32_t*>(og + static_cast<long long>(row_a) * p.o_stride + col) =
          pack2(o[n][0] * inv0, o[n][1] * inv0);
    if (row_b < p.S)
      *reinterpret_cast<uint32_t*>(og + static_cast<long long>(row_b) * p.o_stride + col) =
          pack2(o[n][2] * inv1, o[n][3] * inv1);
  }
  if (t4 == 0) {
    float* lse = p.lse + (static_cast<long long>(b) * p.Hq + h) * p.S;
    if (row_a < p.S) lse[row_a] = (l_r[0] > 0.f) ? (m_r[0] * p.scale + logf(l_r[0])) : INFINITY;
    if (row_b < p.S) lse[row_b] = (l_r[1] > 0.f) ? (m_r[1] * p.scale + logf(l_r[1])) : INFINITY;
  }
}

// ------------------------------------------------------------------------------------------ backward
// delta[b, h, s] = sum_d dO[b s, h d] * O[b s, h d]
template <int D>
__global__ void attn_bwd_delta_kernel(AttnBwdArgs p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(p.B) * p.S * p.Hq;
  if (warp >= total) return;
  const int h = warp % p.Hq;
  const long long row = warp / p.Hq;  // b * S + s
  const int b = row / p.S, s = row % p.S;
  const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(p.o) + row * p.o_stride + h * D;
  const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(p.dout) + row * p.do_stride + h * D;
  float acc = 0.f;
  for (int c = lane * 2; c < D; c += 64) {
    const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(o + c));
    const float2 e = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(d + c));
    acc += a.x * e.x + a.y * e.y;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) p.delta[(static_cast<long long>(b) * p.Hq + h) * p.S + s] = acc;
}

// dK, dV for BN = 16 * WARPS key rows of one (b, kv head); loops over the q heads of the group
// and over q blocks of BMq rows.
template <int D, int WARPS, int BMQ>
__global__ void __launch_bounds__(WARPS * 32) attn_bwd_dkdv_kernel(AttnBwdArgs p) {
  constexpr int BN = 16 * WARPS;
  constexpr int THREADS = WARPS * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BN * D * 2;
  const uint32_t sQ = sV + BN * D * 2;          // 2 buffers
  const uint32_t sdO = sQ + 2 * BMQ * D * 2;    // 2 buffers
  float* sLse = reinterpret_cast<float*>(smem + (2 * BN + 4 * BMQ) * D * 2);  // 2 x BMQ
  float* sDelta = sLse + 2 * BMQ;

  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int group = p.Hq / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int k0 = kb * BN;
  const long long boff_k = static_cast<long long>(b) * p.S;
  const __nv_bfloat16* kg = reinterpret_cast<const __nv_bfloat16*>(p.k) + boff_k * p.k_stride + hk * D;
  const __nv_bfloat16* vg = reinterpret_cast<const __nv_bfloat16*>(p.v) + boff_k * p.v_stride + hk * D;

  load_tile<BN, D, THREADS>(sK, kg, p.k_stride, k0, p.S);
  load_tile<BN, D, THREADS>(sV, vg, p.v_stride, k0, p.S);
  cp_commit();
  cp_wait<0>();
  __syncthreads();

  const int arow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // A-fragment row of this lane
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const float sl2 = p.scale * kLog2e;
  const int qstart_blk = p.causal ? (k0 / BMQ) : 0;
  const int nqb = (p.S + BMQ - 1) / BMQ;
  const int per_head = nqb - qstart_blk;
  const int total = per_head * group;
  const int krow_a = k0 + warp * 16 + g, krow_b = krow_a + 8;

  auto issue = [&](int it, int buf) {
    const int hh = hk * group + it / per_head;
    const int qb = qstart_blk + it % per_head;
    const long long boff = static_cast<long long>(b) * p.S;
    load_tile<BMQ, D, THREADS>(sQ + buf * BMQ * D * 2, reinterpret_cast<const __nv_bfloat16*>(p.q) + boff * p.q_stride + hh * D, p.q_stride, qb * BMQ, p.S);
    load_tile<BMQ, D, THREADS>(sdO + buf * BMQ * D * 2, reinterpret_cast<const __nv_bfloat16*>(p.dout) + boff * p.do_stride + hh * D, p.do_stride,
                               qb * BMQ, p.S);
    const float* lse = p.lse + (static_cast<long long>(b) * p.Hq + hh) * p.S;
    const float* dl = p.delta + (static_cast<long long>(b) * p.Hq + hh) * p.S;
    for (int i = threadIdx.x; i < BMQ; i += THREADS) {
      const int r = qb * BMQ + i;
      sLse[buf * BMQ + i] = (r < p.S) ? lse[r] : INFINITY;
      sDelta[buf * BMQ + i] = (r < p.S) ? dl[r] : 0.f;
    }
  };

  if (total > 0) issue(0, 0);
  cp_commit();
  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    const int qb = qstart_blk + it % per_head;
    const int q0 = qb * BMQ;
    __syncthreads();  // previous iteration done with buf ^ 1
    if (it + 1 < total) issue(it + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t cQ = sQ + buf * BMQ * D * 2, cdO = sdO + buf * BMQ * D * 2;
    const float* cl = sLse + buf * BMQ;
    const float* cd = sDelta + buf * BMQ;

    // S^T[kv, q] and dP^T[kv, q]
    float st[BMQ / 8][4], dpt[BMQ / 8][4];
#pragma unroll
    for (int n = 0; n < BMQ / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[n][e] = dpt[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t kf[4], vf[4];
      ldsm_x4(swz<D>(sK, arow, kk * 16 + (lane >> 4) * 8), kf[0], kf[1], kf[2], kf[3]);
      ldsm_x4(swz<D>(sV, arow, kk * 16 + (lane >> 4) * 8), vf[0], vf[1], vf[2], vf[3]);
#pragma unroll
      for (int n2 = 0; n2 < BMQ / 16; ++n2) {
        const int r = n2 * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(swz<D>(cQ, r, c), b0, b1, b2, b3);
        mma_bf16(st[2 * n2], kf, b0, b1);
        mma_bf16(st[2 * n2 + 1], kf, b2, b3);
        ldsm_x4(swz<D>(cdO, r, c), b0, b1, b2, b3);
        mma_bf16(dpt[2 * n2], vf, b0, b1);
        mma_bf16(dpt[2 * n2 + 1], vf, b2, b3);
      }
    }
    // P^T and dS^T
    uint32_t pf[BMQ / 16][4], dsf[BMQ / 16][4];
#pragma unroll
    for (int n = 0; n < BMQ / 8; ++n) {
      float pv[4], dsv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = n * 8 + t4 * 2 + (e & 1);
        const int qrow = q0 + qi;
        const int krow = (e < 2) ? krow_a : krow_b;
        float x = st[n][e] * sl2 - cl[qi] * kLog2e;
        const bool masked = (qrow >= p.S) || (krow >= p.S) || (p.causal && krow > qrow);
        const float pp = masked ? 0.f : exp2f(x);
        pv[e] = pp;
        dsv[e] = pp * (dpt[n][e] - cd[qi]);
      }
      pf[n >> 1][(n & 1) * 2 + 0] = pack2(pv[0], pv[1]);
      pf[n >> 1][(n & 1) * 2 + 1] = pack2(pv[2], pv[3]);
      dsf[n >> 1][(n & 1) * 2 + 0] = pack2(dsv[0], dsv[1]);
      dsf[n >> 1][(n & 1) * 2 + 1] = pack2(dsv[2], dsv[3]);
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BMQ / 16; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < D / 16; ++n2) {
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = n2 * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(swz<D>(cdO, r, c), b0, b1, b2, b3);
        mma_bf16(dv[2 * n2], pf[kk], b0, b1);
        mma_bf16(dv[2 * n2 + 1], pf[kk], b2, b3);
        ldsm_x4_t(swz<D>(cQ, r, c), b0, b1, b2, b3);
        mma_bf16(dk[2 * n2], dsf[kk], b0, b1);
        mma_bf16(dk[2 * n2 + 1], dsf[kk], b2, b3);
      }
    }
  }
  cp_wait<0>();
  __nv_bfloat16* dkg = reinterpret_cast<__nv_bfloat16*>(p.dk) + static_cast<long long>(b) * p.S * p.dk_stride + hk * D;
  __nv_bfloat16* dvg = reinterpret_cast<__nv_bfloat16*>(p.dv) + static_cast<long long>(b) * p.S * p.dv_stride + hk * D;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + t4 * 2;
    if (krow_a < p.S) {
      *reinterpret_cast<uint32_t*>(dkg + static_cast<long long>(krow_a) * p.dk_stride + col) =
          pack2(dk[n][0] * p.scale, dk[n][1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + static_cast<long long>(krow_a) * p.dv_stride + col) = pack2(dv[n][0], dv[n][1]);
    }
    if (krow_b < p.S) {
      *reinterpret_cast<uint32_t*>(dkg + static_cast<long long>(krow_b) * p.dk_stride + col) =
          pack2(dk[n][2] * p.scale, dk[n][3] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + static_cast<long long>(krow_b) * p.dv_stride + col) = pack2(dv[n][2], dv[n][3]);
    }
  }
}

// dQ for BM = 16 * WARPS query rows of one (b, h); loops over key blocks of BN rows.
template <int D, int WARPS, int BN>
__global__ void __launch_bounds__(WARPS * 32) attn_bwd_dq_kernel(AttnBwdArgs p) {
  constexpr int BM = 16 * WARPS;
  constexpr int THREADS = WARPS * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sdO = sQ + BM * D * 2;
  const uint32_t sK0 = sdO + BM * D * 2;     // 2 buffers
  const uint32_t sV0 = sK0 + 2 * BN * D * 2;  // 2 buffers

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int q0 = qb * BM;
  const long long boff = static_cast<long long>(b) * p.S;
  const __nv_bfloat16* kg = reinterpret_cast<const __nv_bfloat16*>(p.k) + boff * p.k_stride + hk * D;
  const __nv_bfloat16* vg = reinterpret_cast<const __nv_bfloat16*>(p.v) + boff * p.v_stride + hk * D;
  const int kv_end = p.causal ? min(p.S, q0 + BM) : p.S;
  const int nkb = (kv_end + BN - 1) / BN;

  load_tile<BM, D, THREADS>(sQ, reinterpret_cast<const __nv_bfloat16*>(p.q) + boff * p.q_stride + h * D, p.q_stride, q0, p.S);
  load_tile<BM, D, THREADS>(sdO, reinterpret_cast<const __nv_bfloat16*>(p.dout) + boff * p.do_stride + h * D, p.do_stride, q0, p.S);
  cp_commit();
  if (nkb > 0) {
    load_tile<BN, D, THREADS>(sK0, kg, p.k_stride, 0, p.S);
    load_tile<BN, D, THREADS>(sV0, vg, p.v_stride, 0, p.S);
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();

  const int arow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int row_a = q0 + warp * 16 + g, row_b = row_a + 8;
  const float* lse = p.lse + (static_cast<long long>(b) * p.Hq + h) * p.S;
  const float* dl = p.delta + (static_cast<long long>(b) * p.Hq + h) * p.S;
  const float l2a = (row_a < p.S) ? lse[row_a] * kLog2e : INFINITY;
  const float l2b = (row_b < p.S) ? lse[row_b] * kLog2e : INFINITY;
  const float da = (row_a < p.S) ? dl[row_a] : 0.f;
  const float db = (row_b < p.S) ? dl[row_b] : 0.f;
  const float sl2 = p.scale * kLog2e;

  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    const uint32_t sK = sK0 + buf * BN * D * 2, sV = sV0 + buf * BN * D * 2;
    if (j + 1 < nkb) {
      load_tile<BN, D, THREADS>(sK0 + (buf ^ 1) * BN * D * 2, kg, p.k_stride, (j + 1) * BN, p.S);
      load_tile<BN, D, THREADS>(sV0 + (buf ^ 1) * BN * D * 2, vg, p.v_stride, (j + 1) * BN, p.S);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t qf[4], dof[4];
      ldsm_x4(swz<D>(sQ, arow, kk * 16 + (lane >> 4) * 8), qf[0], qf[1], qf[2], qf[3]);
      ldsm_x4(swz<D>(sdO, arow, kk * 16 + (lane >> 4) * 8), dof[0], dof[1], dof[2], dof[3]);
#pragma unroll
      for (int n2 = 0; n2 < BN / 16; ++n2) {
        const int r = n2 * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(swz<D>(sK, r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * n2], qf, b0, b1);
        mma_bf16(s[2 * n2 + 1], qf, b2, b3);
        ldsm_x4(swz<D>(sV, r, c), b0, b1, b2, b3);
        mma_bf16(dp[2 * n2], dof, b0, b1);
        mma_bf16(dp[2 * n2 + 1], dof, b2, b3);
      }
    }
    const int kbase = j * BN;
    uint32_t dsf[BN / 16][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      float dsv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = kbase + n * 8 + t4 * 2 + (e & 1);
        const int row = (e < 2) ? row_a : row_b;
        const bool masked = (col >= p.S) || (row >= p.S) || (p.causal && col > row);
        const float pp = masked ? 0.f : exp2f(s[n][e] * sl2 - ((e < 2) ? l2a : l2b));
        dsv[e] = pp * (dp[n][e] - ((e < 2) ? da : db));
      }
      dsf[n >> 1][(n & 1) * 2 + 0] = pack2(dsv[0], dsv[1]);
      dsf[n >> 1][(n & 1) * 2 + 1] = pack2(dsv[2], dsv[3]);
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < D / 16; ++n2) {
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = n2 * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(swz<D>(sK, r, c), b0, b1, b2, b3);
        mma_bf16(dq[2 * n2], dsf[kk], b0, b1);
        mma_bf16(dq[2 * n2 + 1], dsf[kk], b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  __nv_bfloat16* dqg = reinterpret_cast<__nv_bfloat16*>(p.dq) + boff * p.dq_stride + h * D;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + t4 * 2;
    if (row_a < p.S)
      *reinterpret_cast<uint32_t*>(dqg + static_cast<long long>(row_a) * p.dq_stride + col) =
          pack2(dq[n][0] * p.scale, dq[n][1] * p.scale);
    if (row_b < p.S)
      *reinterpret_cast<uint32_t*>(dqg + static_cast<long long>(row_b) * p.dq_stride + col) =
          pack2(dq[n][2] * p.scale, dq[n][3] * p.scale);
  }
}

template <typename K>
int set_smem(K kern, int bytes) {
  return static_cast<int>(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <int D>
int fwd_impl(const AttnArgs& a, cudaStream_t s) {
  constexpr int WARPS = 8, BN = 64, BM = 16 * WARPS;
  const int smem = (BM + 4 * BN) * D * 2;
  auto kern = attn_fwd_kernel<D, WARPS, BN>;
  if (int e = set_smem(kern, smem)) return e;
  dim3 grid((a.S + BM - 1) / BM, a.Hq, a.B);
  kern<<<grid, WARPS * 32, smem, s>>>(a);
  return static_cast<int>(cudaGetLastError());
}

template <int D>
int bwd_impl(const AttnBwdArgs& a, cudaStream_t s) {
  {
    const long long warps = static_cast<long long>(a.B) * a.S * a.Hq;
    const int blocks = static_cast<int>((warps * 32 + 255) / 256);
    attn_bwd_delta_kernel<D><<<blocks, 256, 0, s>>>(a);
  }
  {
    constexpr int WARPS = 4, BMQ = 32, BN = 16 * WARPS;
    const int smem = (2 * BN + 4 * BMQ) * D * 2 + 4 * BMQ * 4;
    auto kern = attn_bwd_dkdv_kernel<D, WARPS, BMQ>;
    if (int e = set_smem(kern, smem)) return e;
    dim3 grid((a.S + BN - 1) / BN, a.Hkv, a.B);
    kern<<<grid, WARPS * 32, smem, s>>>(a);
  }
  {
    constexpr int WARPS = 4, BN = 64, BM = 16 * WARPS;
    const int smem = (2 * BM + 4 * BN) * D * 2;
    auto kern = attn_bwd_dq_kernel<D, WARPS, BN>;
    if (int e = set_smem(kern, smem)) return e;
    dim3 grid((a.S + BM - 1) / BM, a.Hq, a.B);
    kern<<<grid, WARPS * 32, smem, s>>>(a);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

int attention_fwd_mma(const AttnArgs& a, int D, cudaStream_t s) {
  if (a.Hq % a.Hkv) return -1;
  if (D == 128) return fwd_impl<128>(a, s);
  if (D == 64) return fwd_impl<64>(a, s);
  return -2;
}

int attention_bwd_mma(const AttnBwdArgs& a, int D, cudaStream_t s) {
  if (a.Hq % a.Hkv) return -1;
  if (D == 128) return bwd_impl<128>(a, s);
  if (D == 64) return bwd_impl<64>(a, s);
  return -2;
}

}  // namespace rb
