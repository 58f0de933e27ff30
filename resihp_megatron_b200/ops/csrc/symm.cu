// Symmetric peer memory for one generation of ranks on one NVLink/NVSwitch node, and the
// kernels that use it.
//
// * Heap: each rank cudaMallocs one region, exports a CUDA IPC handle, and maps every peer's
//   region (cudaIpcOpenMemHandle); a generation change unmaps and rebuilds.  The first
//   kSignalBytes of every region are a signal pad: slot p (one 64-bit word per rank, on its own
//   128-byte line) is written only by rank p.
// * Abort word: pinned, host-mapped memory.  The control plane sets it from the host while a
//   kernel runs; every spin-wait below polls it and returns with an error status.
// * Barrier kernel: rank r stores `epoch` into slot r of every peer's pad (release, system
//   scope, after a system fence so all earlier writes of this rank are visible), then waits --
//   bounded by %globaltimer -- until every slot of its own pad reaches `epoch`.  Runs as one
//   block; ranks are different GPUs, so the waiting kernels always run concurrently.
// * Fused data-parallel step: rank r owns a contiguous shard of the flat parameter space.  One
//   kernel sums the shard's fp32 gradients over all ranks with peer loads in rank order (fixed
//   order: deterministic and identical on every rank), applies Adam to the fp32 master shard,
//   and stores the new bf16 weights of the shard into every rank's weight buffer with peer
//   stores: reduce-scatter + optimizer + all-gather in one pass over NVLink, with no
//   intermediate buffers.
//
// Only this file's own kernels touch peer memory; no TMA and no library kernel reads it.
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "kernels.h"
#include "sm100.cuh"

namespace rb {

namespace {

constexpr int kPadStride = 16;  // 64-bit words per signal slot (128 bytes)

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// status[0] = 0 ok, 1 timeout, 2 aborted (sticky until the host clears it); status[1] = the rank
// that was waited for.
__global__ void symm_barrier_kernel(unsigned long long* const* pads, int rank, int world, unsigned long long epoch,
                                    const int* abort_word, int* status, int* err, unsigned long long budget_ns) {
  // A failed barrier is sticky: once one barrier of this heap timed out or was aborted, later
  // ones return at once, so a broken generation costs one budget, not one per barrier, before
  // the host reads the status and raises.
  if (ld_volatile_int(status) != 0) return;
  __threadfence_system();
  __syncthreads();
  const int t = threadIdx.x;
  if (t < world) st_release_sys(pads[t] + rank * kPadStride, epoch);
  __syncthreads();
  if (t < world) {
    const unsigned long long* mine = pads[rank] + t * kPadStride;
    const uint64_t t0 = globaltimer();
    int outcome = 0;
    while (ld_acquire_sys(mine) < epoch) {
      if (abort_word != nullptr && ld_volatile_int(abort_word) != 0) {
        outcome = 2;
        break;
      }
      if (globaltimer() - t0 > budget_ns) {
        outcome = 1;
        break;
      }
      __nanosleep(200);
    }
    if (outcome != 0) {
      if (atomicCAS(status, 0, outcome) == 0) status[1] = t;
      record_error(err, outcome == 1 ? kErrPeerTimeout : kErrAborted);
    }
  }
  __syncthreads();
  __threadfence_system();
}

// ---------------------------------------------------------------- device timing ring
// Host-mapped ring in the NCCL profiler plugin's record format (so detect/nccl_profile_reader
// reads both): header {u32 magic, u32 version, u32 capacity, u32 record size, u64 head}, then
// records {u64 start_ns, u64 end_ns, u64 comm_id, u64 count, i32 rank, i32 nranks, i32 type,
// i32 peer, char func[24], u64 seq}; seq = index + 1 is written last (seqlock).  A kernel that
// reports itself keeps {min start, max end, blocks done} in a device stamp; the last block to
// finish appends one record.
struct RingRecord {
  unsigned long long start_ns, end_ns, comm_id, count;
  int rank, nranks, type, peer;
  char func[24];
  unsigned long long seq;
};

struct DevRing {
  unsigned long long* head;  // host-mapped
  RingRecord* records;       // host-mapped
  int capacity, rank, nranks;
};

struct KernelStamp {
  unsigned long long start, end;
  unsigned int done;
  unsigned int pad;
  unsigned long long head;  // records appended so far (device memory: no atomics on host memory)
};

constexpr int kTypeKernel = 1 << 3;

__device__ __forceinline__ void stamp_begin(KernelStamp* st) {
  if (st != nullptr && threadIdx.x == 0) atomicMin(&st->start, static_cast<unsigned long long>(globaltimer()));
}

__device__ void stamp_end(KernelStamp* st, const DevRing& ring, const char (&name)[24], unsigned long long count,
                          unsigned long long comm_id) {
  if (st == nullptr || ring.records == nullptr) return;
  __syncthreads();
  if (threadIdx.x != 0) return;
  atomicMax(&st->end, static_cast<unsigned long long>(globaltimer()));
  __threadfence();
  if (atomicAdd(&st->done, 1u) + 1 != gridDim.x) return;
  // last block: append the record, then reset the stamp for the next launch
  const unsigned long long start = atomicAdd(&st->start, 0ull), end = atomicAdd(&st->end, 0ull);
  const unsigned long long idx = st->head++;  // launches of one stamp are serialised on their stream
  RingRecord* r = ring.records + (idx % static_cast<unsigned long long>(ring.capacity));
  volatile RingRecord* v = r;
  v->seq = 0;
  v->start_ns = start;
  v->end_ns = end;
  v->comm_id = comm_id;
  v->count = count;
  v->rank = ring.rank;
  v->nranks = ring.nranks;
  v->type = kTypeKernel;
  v->peer = -1;
  for (int i = 0; i < 24; ++i) v->func[i] = name[i];
  __threadfence_system();
  v->seq = idx + 1;
  __threadfence_system();
  *reinterpret_cast<volatile unsigned long long*>(ring.head) = idx + 1;  // publish after the record
  st->start = ~0ull;
  st->end = 0;
  st->done = 0;
  __threadfence();
}

constexpr int kMaxWorld = 16;

struct DpStepArgs {
  const float* grads[kMaxWorld];     // every rank's full gradient buffer (peer pointers)
  __nv_bfloat16* weights[kMaxWorld];  // every rank's full bf16 weight buffer (peer pointers)
  float* master;                      // this rank's shard
  float* m;
  float* v;
  long long shard_lo, n;
  int world;
  float lr, b1, b2, eps, wd, bc1, bc2_sqrt, grad_scale;
  int decoupled;
  DevRing ring;
  KernelStamp* stamp;
};

// 4 elements per thread, grid-stride.  Loads of the W gradients are issued together before
// the sum so their NVLink latencies overlap.  The kernel never waits on another rank, so it does
// not poll the abort word (a host-memory read per iteration would cost a PCIe round trip).
__global__ void __launch_bounds__(256) dp_step_kernel(const __grid_constant__ DpStepArgs a) {
  stamp_begin(a.stamp);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 4;
  const float step_size = a.lr / a.bc1;
  for (long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < a.n; i += stride) {
    const long long gi = a.shard_lo + i;
    float4 parts[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < a.world) parts[r] = __ldcv(reinterpret_cast<const float4*>(a.grads[r] + gi));
    float g[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < a.world) {
        g[0] += parts[r].x;
        g[1] += parts[r].y;
        g[2] += parts[r].z;
        g[3] += parts[r].w;
      }
    float4 pp = *reinterpret_cast<const float4*>(a.master + i);
    float4 mm = *reinterpret_cast<const float4*>(a.m + i);
    float4 vv = *reinterpret_cast<const float4*>(a.v + i);
    float* P = &pp.x;
    float* M = &mm.x;
    float* V = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float gj = g[j] * a.grad_scale;
      if (a.wd != 0.f) {
        if (a.decoupled) P[j] *= (1.f - a.lr * a.wd);
        else gj = gj + a.wd * P[j];
      }
      M[j] = M[j] + (1.f - a.b1) * (gj - M[j]);
      V[j] = V[j] * a.b2 + (1.f - a.b2) * gj * gj;
      const float denom = sqrtf(V[j]) / a.bc2_sqrt + a.eps;
      P[j] = P[j] - step_size * (M[j] / denom);
    }
    *reinterpret_cast<float4*>(a.master + i) = pp;
    *reinterpret_cast<float4*>(a.m + i) = mm;
    *reinterpret_cast<float4*>(a.v + i) = vv;
    uint2 u;
    u.x = pack_bf16x2(pp.x, pp.y);
    u.y = pack_bf16x2(pp.z, pp.w);
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < a.world) __stcg(reinterpret_cast<uint2*>(a.weights[r] + gi), u);
  }
  static constexpr char kName[24] = "dp_reduce_adam_gather";
  stamp_end(a.stamp, a.ring, kName, static_cast<unsigned long long>(a.n), 0ull);
}

// Slice migration: every (src, dst, bytes) piece is copied with 16-byte loads and stores; the
// source may be a peer's memory (old generation's heap), the destination is this rank's.  Pieces
// are pre-split on the host to at most kPieceBytes so CTAs share the work evenly.
struct CopyPiece {
  const uint4* src;
  uint4* dst;
  long long n16;  // number of 16-byte units
};

__global__ void __launch_bounds__(256) symm_copy_kernel(const CopyPiece* __restrict__ pieces, int n_pieces) {
  for (int pi = blockIdx.x; pi < n_pieces; pi += gridDim.x) {
    const CopyPiece c = pieces[pi];
    for (long long i = threadIdx.x; i < c.n16; i += blockDim.x * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i + u * blockDim.x < c.n16) v[u] = __ldcv(c.src + i + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i + u * blockDim.x < c.n16) c.dst[i + u * blockDim.x] = v[u];
    }
  }
}

// Strided slice copy: piece = `rows` rows of `row16` 16-byte units, rows `src_pitch16` /
// `dst_pitch16` units apart (a column block of a row-major tensor); pieces are pre-split on the
// host so that each holds at most about 1 MB.
struct CopyPiece2D {
  const uint4* src;
  uint4* dst;
  int rows, row16;
  long long src_pitch16, dst_pitch16;
};

__global__ void __launch_bounds__(256) symm_copy2d_kernel(const CopyPiece2D* __restrict__ pieces, int n_pieces) {
  for (int pi = blockIdx.x; pi < n_pieces; pi += gridDim.x) {
    const CopyPiece2D c = pieces[pi];
    const long long total = static_cast<long long>(c.rows) * c.row16;
    for (long long i = threadIdx.x; i < total; i += blockDim.x * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long g = i + u * blockDim.x;
        if (g < total) {
          const long long r = g / c.row16, q = g - r * c.row16;
          v[u] = __ldcv(c.src + r * c.src_pitch16 + q);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long g = i + u * blockDim.x;
        if (g < total) {
          const long long r = g / c.row16, q = g - r * c.row16;
          c.dst[r * c.dst_pitch16 + q] = v[u];
        }
      }
    }
  }
}

// Rank-ordered sums over peer memory: dst[i] = src[0][i] + src[1][i] + ... (fp32, in the given order,
// so every rank that sums the same sources gets the same bits).  The piece table stays on the
// device between launches.
constexpr int kSumMaxSrc = 8;
struct SumPiece {
  float* dst;
  const float* src[kSumMaxSrc];
  long long n;
  int nsrc;
  int vec4;  // n % 4 == 0 and every pointer 16-byte aligned
};

__global__ void __launch_bounds__(256) symm_sum_kernel(const SumPiece* __restrict__ pieces, int n_pieces) {
  for (int pi = blockIdx.x; pi < n_pieces; pi += gridDim.x) {
    const SumPiece p = pieces[pi];
    if (p.vec4) {
      const long long n4 = p.n / 4;
      for (long long i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 acc = __ldcv(reinterpret_cast<const float4*>(p.src[0]) + i);
        for (int k = 1; k < p.nsrc; ++k) {
          const float4 v = __ldcv(reinterpret_cast<const float4*>(p.src[k]) + i);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        reinterpret_cast<float4*>(p.dst)[i] = acc;
      }
    } else {
      for (long long i = threadIdx.x; i < p.n; i += blockDim.x) {
        float acc = __ldcv(p.src[0] + i);
        for (int k = 1; k < p.nsrc; ++k) acc += __ldcv(p.src[k] + i);
        p.dst[i] = acc;
      }
    }
  }
}

// All-gather of equal row chunks: chunk c of `dst` (this rank's buffer) is filled from `src[c]`
// (chunk c in rank c's buffer) for every c != self; the work is cut into 1 MB slices spread over
// the grid.  No piece table, so nothing is staged on the host.
struct GatherArgs {
  const uint4* src[kMaxWorld];
  uint4* dst;
  long long chunk16;
  int world, self;
};

__global__ void __launch_bounds__(256) symm_gather_kernel(GatherArgs a) {
  constexpr long long kSlice16 = (1 << 20) / 16;
  const long long per_chunk = (a.chunk16 + kSlice16 - 1) / kSlice16;
  const long long slices = per_chunk * (a.world - 1);
  for (long long sl = blockIdx.x; sl < slices; sl += gridDim.x) {
    const int k = static_cast<int>(sl / per_chunk);
    const int c = (a.self + 1 + k) % a.world;
    const long long lo = (sl - k * per_chunk) * kSlice16;
    const long long hi = lo + kSlice16 < a.chunk16 ? lo + kSlice16 : a.chunk16;
    const uint4* src = a.src[c];
    uint4* dst = a.dst + c * a.chunk16;
    for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i + u * blockDim.x < hi) v[u] = __ldcv(src + i + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i + u * blockDim.x < hi) dst[i + u * blockDim.x] = v[u];
    }
  }
}

}  // namespace

// ----------------------------------------------------------------------------------- host side
int symm_signal_bytes(int world) { return world * kPadStride * 8; }

int symm_gather(const void* const* src, void* dst, long long chunk_bytes, int world, int self, int num_sms,
                cudaStream_t s) {
  if (world < 1 || world > kMaxWorld || self < 0 || self >= world || (chunk_bytes & 15) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return -1;
  if (world == 1 || chunk_bytes == 0) return 0;
  GatherArgs a{};
  for (int c = 0; c < world; ++c) {
    if (reinterpret_cast<uintptr_t>(src[c]) & 15) return -1;
    a.src[c] = reinterpret_cast<const uint4*>(src[c]);
  }
  a.dst = reinterpret_cast<uint4*>(dst);
  a.chunk16 = chunk_bytes / 16;
  a.world = world;
  a.self = self;
  const long long slices = ((a.chunk16 + (1 << 16) - 1) >> 16) * (world - 1);
  const int grid = slices < num_sms * 4 ? static_cast<int>(slices) : num_sms * 4;
  symm_gather_kernel<<<grid, 256, 0, s>>>(a);
  return static_cast<int>(cudaGetLastError());
}

int symm_barrier(unsigned long long* const* pads_dev, int rank, int world, unsigned long long epoch,
                 const int* abort_word, int* status, int* err, double budget_s, cudaStream_t s) {
  if (world < 1 || world > 1024 || rank < 0 || rank >= world) return -1;
  const int threads = ((world + 31) / 32) * 32;
  symm_barrier_kernel<<<1, threads, 0, s>>>(pads_dev, rank, world, epoch, abort_word, status, err,
                                            static_cast<unsigned long long>(budget_s * 1e9));
  return static_cast<int>(cudaGetLastError());
}

int dp_step_fused(const float* const* grads, __nv_bfloat16* const* weights, int world, float* master, float* m,
                  float* v, long long shard_lo, long long n, float lr, float b1, float b2, float eps, float wd,
                  int decoupled, float bc1, float bc2_sqrt, float grad_scale, const int* abort_word, int num_sms,
                  cudaStream_t s, void* ring_base, int ring_capacity, void* stamp) {
  if (world < 1 || world > kMaxWorld || (n & 3) || (shard_lo & 3)) return -1;
  DpStepArgs a{};
  for (int r = 0; r < world; ++r) {
    a.grads[r] = grads[r];
    a.weights[r] = weights[r];
    if ((reinterpret_cast<uintptr_t>(grads[r]) & 15) || (reinterpret_cast<uintptr_t>(weights[r]) & 7)) return -2;
  }
  if ((reinterpret_cast<uintptr_t>(master) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15)
    return -2;
  a.master = master;
  a.m = m;
  a.v = v;
  a.shard_lo = shard_lo;
  a.n = n;
  a.world = world;
  a.lr = lr;
  a.b1 = b1;
  a.b2 = b2;
  a.eps = eps;
  a.wd = wd;
  a.decoupled = decoupled;
  a.bc1 = bc1;
  a.bc2_sqrt = bc2_sqrt;
  a.grad_scale = grad_scale;
  (void)abort_word;  // no waits inside: see dp_step_kernel
  // ring header: u32 magic, version, capacity, record size, u64 head (offset 16); records at 24
  a.ring.head = ring_base != nullptr ? reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(ring_base) + 16)
                                     : nullptr;
  a.ring.records = ring_base != nullptr ? reinterpret_cast<RingRecord*>(static_cast<uint8_t*>(ring_base) + 24) : nullptr;
  a.ring.capacity = ring_capacity;
  a.ring.rank = 0;
  a.ring.nranks = world;
  a.stamp = reinterpret_cast<KernelStamp*>(stamp);
  const long long threads_needed = n / 4;
  long long blocks = (threads_needed + 255) / 256;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  dp_step_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(a);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rb

namespace rb {

// pieces: host array of (src, dst, bytes) triples, each 16-byte aligned; `dev_scratch` holds at
// least `max_pieces` CopyPiece records on the device.
int symm_copy(const long long* triples, int n, void* dev_scratch, int max_pieces, int num_sms, cudaStream_t s) {
  constexpr long long kPieceBytes = 1 << 20;
  std::vector<CopyPiece> pieces;
  for (int i = 0; i < n; ++i) {
    const long long src = triples[3 * i], dst = triples[3 * i + 1], bytes = triples[3 * i + 2];
    if ((src | dst | bytes) & 15) return -1;
    for (long long off = 0; off < bytes; off += kPieceBytes) {
      const long long b = bytes - off < kPieceBytes ? bytes - off : kPieceBytes;
      pieces.push_back({reinterpret_cast<const uint4*>(src + off), reinterpret_cast<uint4*>(dst + off), b / 16});
    }
  }
  if (pieces.empty()) return 0;
  if (static_cast<int>(pieces.size()) > max_pieces) return -2;
  cudaError_t e = cudaMemcpyAsync(dev_scratch, pieces.data(), pieces.size() * sizeof(CopyPiece),
                                  cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return static_cast<int>(e);
  // the host vector must outlive the async copy: wait for it on the stream before returning
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return static_cast<int>(e);
  const int grid = static_cast<int>(pieces.size()) < num_sms * 4 ? static_cast<int>(pieces.size()) : num_sms * 4;
  symm_copy_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const CopyPiece*>(dev_scratch),
                                        static_cast<int>(pieces.size()));
  return static_cast<int>(cudaGetLastError());
}

int symm_copy_piece_bytes() { return static_cast<int>(sizeof(CopyPiece)); }

// pieces: host array of (src, dst, rows, row_bytes, src_pitch, dst_pitch) sextuples, addresses,
// row bytes and pitches 16-byte aligned; `dev_scratch` holds at least `max_pieces` records.
int symm_copy2d(const long long* six, int n, void* dev_scratch, int max_pieces, int num_sms, cudaStream_t s) {
  constexpr long long kPieceBytes = 1 << 20;
  std::vector<CopyPiece2D> pieces;
  for (int i = 0; i < n; ++i) {
    const long long src = six[6 * i], dst = six[6 * i + 1], rows = six[6 * i + 2], row_bytes = six[6 * i + 3];
    const long long sp = six[6 * i + 4], dp = six[6 * i + 5];
    if ((src | dst | row_bytes | sp | dp) & 15) return -1;
    if (rows <= 0 || row_bytes <= 0) continue;
    if (row_bytes > kPieceBytes) {  // long rows: one piece per (row, 1 MB column block)
      for (long long r = 0; r < rows; ++r)
        for (long long off = 0; off < row_bytes; off += kPieceBytes) {
          const long long b = row_bytes - off < kPieceBytes ? row_bytes - off : kPieceBytes;
          pieces.push_back({reinterpret_cast<const uint4*>(src + r * sp + off),
                            reinterpret_cast<uint4*>(dst + r * dp + off), 1, static_cast<int>(b / 16), 0, 0});
        }
      continue;
    }
    const long long per = kPieceBytes / row_bytes;  // rows per piece (>= 1)
    for (long long r = 0; r < rows; r += per) {
      const long long nr = rows - r < per ? rows - r : per;
      pieces.push_back({reinterpret_cast<const uint4*>(src + r * sp), reinterpret_cast<uint4*>(dst + r * dp),
                        static_cast<int>(nr), static_cast<int>(row_bytes / 16), sp / 16, dp / 16});
    }
  }
  if (pieces.empty()) return 0;
  if (static_cast<int>(pieces.size()) > max_pieces) return -2;
  cudaError_t e = cudaMemcpyAsync(dev_scratch, pieces.data(), pieces.size() * sizeof(CopyPiece2D),
                                  cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaStreamSynchronize(s);  // the host vector must outlive the copy
  if (e != cudaSuccess) return static_cast<int>(e);
  const int grid = static_cast<int>(pieces.size()) < num_sms * 4 ? static_cast<int>(pieces.size()) : num_sms * 4;
  symm_copy2d_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const CopyPiece2D*>(dev_scratch),
                                          static_cast<int>(pieces.size()));
  return static_cast<int>(cudaGetLastError());
}

// Resident piece tables: built once (host -> device copy, one synchronisation), launched many times.
int symm_copy2d_build(const long long* six, int n, void* dev_table, int max_pieces, int* count, cudaStream_t s) {
  constexpr long long kPieceBytes = 1 << 20;
  std::vector<CopyPiece2D> pieces;
  for (int i = 0; i < n; ++i) {
    const long long src = six[6 * i], dst = six[6 * i + 1], rows = six[6 * i + 2], row_bytes = six[6 * i + 3];
    const long long sp = six[6 * i + 4], dp = six[6 * i + 5];
    if ((src | dst | row_bytes | sp | dp) & 15) return -1;
    if (rows <= 0 || row_bytes <= 0) continue;
    if (row_bytes > kPieceBytes) {
      for (long long r = 0; r < rows; ++r)
        for (long long off = 0; off < row_bytes; off += kPieceBytes) {
          const long long b = row_bytes - off < kPieceBytes ? row_bytes - off : kPieceBytes;
          pieces.push_back({reinterpret_cast<const uint4*>(src + r * sp + off),
                            reinterpret_cast<uint4*>(dst + r * dp + off), 1, static_cast<int>(b / 16), 0, 0});
        }
      continue;
    }
    const long long per = kPieceBytes / row_bytes;
    for (long long r = 0; r < rows; r += per) {
      const long long nr = rows - r < per ? rows - r : per;
      pieces.push_back({reinterpret_cast<const uint4*>(src + r * sp), reinterpret_cast<uint4*>(dst + r * dp),
                        static_cast<int>(nr), static_cast<int>(row_bytes / 16), sp / 16, dp / 16});
    }
  }
  *count = static_cast<int>(pieces.size());
  if (pieces.empty()) return 0;
  if (static_cast<int>(pieces.size()) > max_pieces) return -2;
  cudaError_t e = cudaMemcpyAsync(dev_table, pieces.data(), pieces.size() * sizeof(CopyPiece2D),
                                  cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaStreamSynchronize(s);
  return static_cast<int>(e);
}

int symm_copy2d_run(const void* dev_table, int count, int num_sms, cudaStream_t s) {
  if (count <= 0) return 0;
  const int grid = count < num_sms * 4 ? count : num_sms * 4;
  symm_copy2d_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const CopyPiece2D*>(dev_table), count);
  return static_cast<int>(cudaGetLastError());
}

int symm_sum_piece_bytes() { return static_cast<int>(sizeof(SumPiece)); }

// entries: per piece (dst, n, nsrc, src[0..7]) as 11 long longs; pieces are split into 1 MB runs.
int symm_sum_build(const long long* entries, int n, void* dev_table, int max_pieces, int* count, cudaStream_t s) {
  constexpr long long kRun = (1 << 20) / 4;
  std::vector<SumPiece> pieces;
  for (int i = 0; i < n; ++i) {
    const long long* e = entries + 11 * i;
    const long long len = e[1];
    const int nsrc = static_cast<int>(e[2]);
    if (len <= 0) continue;
    if (nsrc < 1 || nsrc > kSumMaxSrc) return -1;
    for (long long off = 0; off < len; off += kRun) {
      SumPiece p{};
      p.dst = reinterpret_cast<float*>(e[0]) + off;
      p.n = len - off < kRun ? len - off : kRun;
      p.nsrc = nsrc;
      uintptr_t bits = reinterpret_cast<uintptr_t>(p.dst);
      for (int k = 0; k < nsrc; ++k) {
        p.src[k] = reinterpret_cast<const float*>(e[3 + k]) + off;
        bits |= reinterpret_cast<uintptr_t>(p.src[k]);
      }
      p.vec4 = (p.n % 4 == 0) && (bits & 15) == 0;
      pieces.push_back(p);
    }
  }
  *count = static_cast<int>(pieces.size());
  if (pieces.empty()) return 0;
  if (static_cast<int>(pieces.size()) > max_pieces) return -2;
  cudaError_t e = cudaMemcpyAsync(dev_table, pieces.data(), pieces.size() * sizeof(SumPiece), cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaStreamSynchronize(s);
  return static_cast<int>(e);
}

int symm_sum_run(const void* dev_table, int count, int num_sms, cudaStream_t s) {
  if (count <= 0) return 0;
  const int grid = count < num_sms * 4 ? count : num_sms * 4;
  symm_sum_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const SumPiece*>(dev_table), count);
  return static_cast<int>(cudaGetLastError());
}

long long symm_sum_pieces(const long long* entries, int n) {
  constexpr long long kRun = (1 << 20) / 4;
  long long count = 0;
  for (int i = 0; i < n; ++i) {
    const long long len = entries[11 * i + 1];
    if (len > 0) count += (len + kRun - 1) / kRun;
  }
  return count;
}

long long symm_copy2d_pieces(const long long* six, int n) {
  constexpr long long kPieceBytes = 1 << 20;
  long long count = 0;
  for (int i = 0; i < n; ++i) {
    const long long rows = six[6 * i + 2], row_bytes = six[6 * i + 3];
    if (rows <= 0 || row_bytes <= 0) continue;
    if (row_bytes > kPieceBytes) count += rows * ((row_bytes + kPieceBytes - 1) / kPieceBytes);
    else count += (rows + kPieceBytes / row_bytes - 1) / (kPieceBytes / row_bytes);
  }
  return count;
}

int symm_copy2d_piece_bytes() { return static_cast<int>(sizeof(CopyPiece2D)); }

namespace {
// Reduce-scatter finish: out[i] = sum over slots s (rank order) of recv[s][i], fp32 accumulate.
__global__ void rs_reduce_kernel(const __nv_bfloat16* __restrict__ recv, int world, long long n,
                                 __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ residual) {
  const long long i8 = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i8 >= n) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (residual != nullptr) {  // residual added first, then the slots in rank order
    const uint4 u = *reinterpret_cast<const uint4*>(residual + i8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      acc[2 * j] = f.x;
      acc[2 * j + 1] = f.y;
    }
  }
  for (int s = 0; s < world; ++s) {
    const uint4 u = __ldcv(reinterpret_cast<const uint4*>(recv + s * n + i8));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      acc[2 * j] += f.x;
      acc[2 * j + 1] += f.y;
    }
  }
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(out + i8) = o;
}
}  // namespace

int rs_reduce(const void* recv, int world, long long n, void* out, const void* residual, cudaStream_t s) {
  if ((n & 7) || ((reinterpret_cast<uintptr_t>(recv) | reinterpret_cast<uintptr_t>(out) |
                   reinterpret_cast<uintptr_t>(residual)) & 15))
    return -1;
  const long long threads = n / 8;
  rs_reduce_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(recv), world, n, reinterpret_cast<__nv_bfloat16*>(out),
      reinterpret_cast<const __nv_bfloat16*>(residual));
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rb

namespace rb {
int ring_record_bytes() { return static_cast<int>(sizeof(RingRecord)); }
int kernel_stamp_bytes() { return static_cast<int>(sizeof(KernelStamp)); }
}  // namespace rb
