// Host-side entry points of the sm_100a kernels (implemented in the *.cu files of this
// directory).  All functions return 0 on success; negative values flag bad arguments and
// positive values are CUDA error codes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace rb {

int gemm_bf16(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* D,
              long long ldd, const void* R, long long ldr, int M, int N, int K, int epi, float alpha,
              int* err, int num_sms, cudaStream_t stream, int variant = 0, void* split_ws = nullptr, int splits = 1,
              int split_full = 0);
// Split-K plan of the CTA-pair GEMM (shares per split tile, 1 = none; `*full` leading tiles run
// whole) and the workspace bytes a split launch needs.
int gemm_pair_splits(int M, int N, int K, int variant, int num_sms, int* full);
long long gemm_split_ws_bytes(int M, int N, int splits, int full);

int rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int T, int H, float eps, cudaStream_t s);
int rmsnorm_bwd_blocks(int T);
// RMSNorm whose output is written as block-scaled fp8 (1 x 128 row blocks; scale of block cb of
// row t at s[cb * s_kb + t * s_row]); bit-identical to rmsnorm_fwd followed by fp8_quantize.
// MLP activation (GELU of [T, F], or SwiGLU of [T, 2F]) written as block-scaled fp8 [T, F]; bit-identical
// to gelu_fwd / swiglu_fwd followed by fp8_quantize.
int act_fp8(const void* in, int gated, int T, int F, int fmt, void* q, float* s, long long s_kb, long long s_row,
            unsigned int* amax, cudaStream_t st);
int rmsnorm_fp8(const void* x, const void* w, float* rstd, int T, int H, float eps, int fmt, void* q, float* s,
                long long s_kb, long long s_row, unsigned int* amax, cudaStream_t st);
int rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, const void* dres, void* dx,
                float* dw, int accumulate, float* part, int T, int H, cudaStream_t s);
int rope_apply(void* q, long long row_stride, int heads, int D, const float* cos_t, const float* sin_t, int S,
               int T, int inverse, cudaStream_t s);
int swiglu_fwd(const void* gu, void* a, int T, int F, cudaStream_t s);
int swiglu_bwd(const void* gu, const void* da, void* dgu, int T, int F, cudaStream_t s);
int gelu_fwd(const void* h, void* a, long long n, cudaStream_t s);
int amax_history_push(float* hist, float* pending, int n, int len, cudaStream_t s);
int gelu_bwd(const void* h, const void* da, void* dh, long long n, cudaStream_t s);
int embedding_fwd(const int64_t* ids, const void* E, void* x, int T, int H, int V, int* err, cudaStream_t s);
int embedding_bwd(const int64_t* vals, const int64_t* order, int T, const void* dx, float* dE, int H,
                  cudaStream_t s);
int adam_step(float* p, float* grad, float* m, float* v, void* p_bf16, long long n, float lr, float b1, float b2,
              float eps, float wd, int decoupled, float bc1, float bc2_sqrt, float grad_scale, int zero_grad,
              cudaStream_t s,
              const float* bc_dev = nullptr);
int sumsq_partial(const float* x, long long n, float* part, int nblocks, cudaStream_t s);
int cross_entropy_fwd_bwd(void* logits, long long ld, const int64_t* labels, float* loss, float* lse, int T, int V,
                          long long v0, float grad_scale, long long ignore_index, int write_grad, cudaStream_t s);

struct AttnArgs;
struct AttnBwdArgs;

}  // namespace rb

// Attention argument blocks (shared by the mma.sync and tcgen05 implementations).
namespace rb {
struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  long long q_stride, k_stride, v_stride;
  void* o;
  long long o_stride;
  float* lse;
  int B, S, Hq, Hkv;
  float scale;
  int causal;
};
struct AttnBwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  long long q_stride, k_stride, v_stride, o_stride, do_stride;
  const float* lse;
  float* delta;
  void* dq;
  void* dk;
  void* dv;
  long long dq_stride, dk_stride, dv_stride;
  int B, S, Hq, Hkv;
  float scale;
  int causal;
};
int attention_fwd_mma(const AttnArgs& a, int D, cudaStream_t s);
int attention_fwd_sm100(const AttnArgs& a, int D, int* err, cudaStream_t s, int variant = -1);
int attention_bwd_mma(const AttnBwdArgs& a, int D, cudaStream_t s);
// Symmetric peer memory (symm.cu).
int symm_signal_bytes(int world);
int symm_barrier(unsigned long long* const* pads_dev, int rank, int world, unsigned long long epoch,
                 const int* abort_word, int* status, int* err, double budget_s, cudaStream_t s);
int dp_step_fused(const float* const* grads, __nv_bfloat16* const* weights, int world, float* master, float* m,
                  float* v, long long shard_lo, long long n, float lr, float b1, float b2, float eps, float wd,
                  int decoupled, float bc1, float bc2_sqrt, float grad_scale, const int* abort_word, int num_sms,
                  cudaStream_t s, void* ring_base = nullptr, int ring_capacity = 0, void* stamp = nullptr);
int ring_record_bytes();
// cuMem regions shared as POSIX file descriptors (vmm_heap.cu).
int vmm_available();
long long vmm_round(int device, long long bytes);
int vmm_alloc(int device, long long bytes, void** ptr, int* fd);
int vmm_import(int device, int fd, long long bytes, void** ptr);
int vmm_free(void* ptr);
int kernel_stamp_bytes();
int symm_copy(const long long* triples, int n, void* dev_scratch, int max_pieces, int num_sms, cudaStream_t s);
// All-gather of equal chunks from peers' buffers into this rank's buffer (no host staging).
int symm_gather(const void* const* src, void* dst, long long chunk_bytes, int world, int self, int num_sms,
                cudaStream_t s);
// Strided slice copies (rows x row_bytes with source / destination pitches), pre-split on the host.
int symm_copy2d(const long long* six, int n, void* dev_scratch, int max_pieces, int num_sms, cudaStream_t s);
long long symm_copy2d_pieces(const long long* six, int n);
// Resident piece tables (built once, launched per step): strided copies and rank-ordered fp32 sums.
int symm_copy2d_build(const long long* six, int n, void* dev_table, int max_pieces, int* count, cudaStream_t s);
int symm_copy2d_run(const void* dev_table, int count, int num_sms, cudaStream_t s);
int symm_sum_piece_bytes();
long long symm_sum_pieces(const long long* entries, int n);
int symm_sum_build(const long long* entries, int n, void* dev_table, int max_pieces, int* count, cudaStream_t s);
int symm_sum_run(const void* dev_table, int count, int num_sms, cudaStream_t s);
int symm_copy2d_piece_bytes();
int symm_copy_piece_bytes();
int rs_reduce(const void* recv, int world, long long n, void* out, const void* residual, cudaStream_t s);
// Expert parallelism (moe.cu).
int moe_route(const void* x, const void* w, const float* bias, int T, int H, int E, int k, float* logits, int* topi,
              float* gates, cudaStream_t s);
int moe_positions(const int* topi, int n, int E, int* pos, int* counts, cudaStream_t s);
int moe_dispatch(const void* x, const int* topi, const int* pos, int T, int k, int H, int world, int me, int E,
                 const int* period, const int* cycle, const int* cycle_rank, const int* per_cycle,
                 const long long* rowbase, void* const* recv, long long* route_row, cudaStream_t s);
int moe_combine(const void* residual, const float* gates, const long long* route_row, int T, int k, int H, int world,
                void* const* ybuf, void* out, void* ycache, cudaStream_t s);
int moe_grad_push(const void* dout, const float* gates, const void* ycache, const long long* route_row, int T, int k,
                  int H, int world, void* const* dyrecv, float* dgate, cudaStream_t s);
int moe_grad_pull(const void* dout, const float* gates, const float* dgate, const int* topi,
                  const long long* route_row, int T, int k, int H, int E, int world, void* const* dxbuf, void* dx,
                  float* dlogits, cudaStream_t s, const void* router_w = nullptr);
// Router weight gradient grad [E, H] fp32 += dlogits [T, E]^T x [T, H] (bf16), deterministic;
// `partial` holds moe_router_wgrad_ws_floats(T, H, E) floats.
long long moe_router_wgrad_ws_floats(int T, int H, int E);
int moe_router_wgrad(const float* dlogits, const void* x, int T, int H, int E, float* partial, float* grad,
                     cudaStream_t s);
// Tensor-parallel fused GEMMs (gemm_sm100.cu).
int gemm_ag_bf16(const void* x_full, const void* const* x_src, int world, int self, int chunk_rows, const void* W,
                 bool w_mn, void* Y, int M, int N, int K, int* ready, const int* abort_word, int* err, int num_sms,
                 cudaStream_t stream);
// Words of the `ready` buffer of gemm_ag_bf16 (a work counter and one flag per copy unit).
int gemm_ag_ready_words(int M, int K);
int gemm_rs_scatter_bf16(const void* X, const void* W, bool w_mn, void* const* recv, int world, int slot, int M, int N,
                         int K, int* err, int num_sms, cudaStream_t stream);
// Block-scaled fp8 (fp8_sm100.cu).  fmt: 0 = E4M3, 1 = E5M2.  Scale of operand row r in K-block kb:
// s[kb * kb_stride + (r >> shift) * row_stride] (shift 0: 1 x 128 blocks, 7: 128 x 128 blocks).
int fp8_quantize(const void* x, long long ldx, int R, int C, int fmt, int two_d, void* q_row, float* s_row,
                 void* q_col, float* s_col, unsigned int* amax, cudaStream_t s, int s_row_major = 0, int act = 0);
int gemm_fp8(const void* A, int a_fmt, const void* B, int b_fmt, const float* sa, long long sa_kb, long long sa_row,
             int sa_shift, const float* sb, long long sb_kb, long long sb_row, int sb_shift, void* D, long long ldd,
             int M, int N, int K, int epi, float alpha, int* err, int num_sms, cudaStream_t stream,
             const void* R = nullptr, long long ldr = 0, void* const* rs_dst = nullptr, int world = 0,
             int rs_slot = 0, int variant = 0, void* sf_ws = nullptr);
// Bytes of the packed E8M0 scale words gemm_fp8's block-scaled path (variant 0 / 2) needs as `sf_ws`.
long long gemm_fp8_sf_bytes(int M, int N, int K);
// tcgen05 backward; returns 1 for shapes it does not handle.  `nl2`: B * Hq * S floats of scratch.
int attention_bwd_sm100(const AttnBwdArgs& a, int D, float* nl2, int* err, cudaStream_t s, int variant = -1);
}  // namespace rb
