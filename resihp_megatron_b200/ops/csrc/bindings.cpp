// Python bindings of the sm_100a kernels.  Kernel files (*.cu) include no torch headers;
// this file turns tensors into raw pointers, picks the current stream and reports errors.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <unordered_map>

#include "kernels.h"

namespace {

// One error word per device, written by kernels whose bounded waits ran out.
torch::Tensor& error_word(int device) {
  static std::mutex mu;
  static std::unordered_map<int, torch::Tensor> words;
  std::lock_guard<std::mutex> g(mu);
  auto it = words.find(device);
  if (it == words.end()) {
    auto t = torch::zeros({4}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, device));
    it = words.emplace(device, t).first;
  }
  return it->second;
}

int* err_ptr(const torch::Tensor& like) { return error_word(like.get_device()).data_ptr<int>(); }

int num_sms(int device) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  cache[device] = n;
  return n;
}

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// Leading dimension of a 2-D operand whose inner dimension is contiguous.
long long ld_of(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have a contiguous inner dimension");
  return t.size(0) > 1 ? t.stride(0) : t.size(1);
}

}  // namespace

// Split-K workspace: one grow-only buffer per (device, stream), so launches on one stream reuse it
// in stream order and launches on different streams never share it.  The map is never destroyed
// (its tensors must not be freed after the CUDA context is gone at exit).
static torch::Tensor split_workspace(const torch::Tensor& like, long long bytes) {
  static std::mutex mu;
  static auto* pool = new std::map<std::pair<int, cudaStream_t>, torch::Tensor>();
  std::lock_guard<std::mutex> lock(mu);
  auto& t = (*pool)[{static_cast<int>(like.get_device()), at::cuda::getCurrentCUDAStream().stream()}];
  if (!t.defined() || t.numel() < bytes) t = torch::empty({bytes}, like.options().dtype(torch::kUInt8));
  return t;
}

// out[M,N] (+)= alpha * op(a) @ op(b)^T ; a is [M,K] (or [K,M] if a_t), b is [N,K] (or [K,N] if b_t)
void gemm(const torch::Tensor& a, bool a_t, const torch::Tensor& b, bool b_t, torch::Tensor& out,
          int64_t epi, double alpha, const c10::optional<torch::Tensor>& residual, int64_t variant) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  check_cuda(out, "out");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16,
              "gemm operands must be bf16");
  const long long lda = ld_of(a, "a"), ldb = ld_of(b, "b"), ldd = ld_of(out, "out");
  const int M = a_t ? a.size(1) : a.size(0);
  const int K = a_t ? a.size(0) : a.size(1);
  const int N = b_t ? b.size(1) : b.size(0);
  const int Kb = b_t ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm: contraction sizes differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: out must be [", M, ", ", N, "]");
  if (epi == 1 || epi == 2) {
    TORCH_CHECK(out.scalar_type() == torch::kFloat32, "fp32 epilogue needs an fp32 output");
  } else {
    TORCH_CHECK(out.scalar_type() == torch::kBFloat16, "bf16 epilogue needs a bf16 output");
  }
  const void* rptr = nullptr;
  long long ldr = 0;
  if (epi == 3) {
    TORCH_CHECK(residual.has_value(), "residual epilogue needs a residual");
    const auto& r = *residual;
    TORCH_CHECK(r.scalar_type() == torch::kBFloat16 && r.size(0) == M && r.size(1) == N, "bad residual");
    rptr = r.data_ptr();
    ldr = ld_of(r, "residual");
  }
  const c10::cuda::CUDAGuard guard(a.device());
  if (K == 0) {
    if (epi == 2) return;
    out.zero_();
    if (epi == 3) out.copy_(*residual);
    return;
  }
  const int sms = num_sms(a.get_device());
  int split_full = 0;
  const int splits = rb::gemm_pair_splits(M, N, K, static_cast<int>(variant), sms, &split_full);
  torch::Tensor ws;
  if (splits > 1) ws = split_workspace(a, rb::gemm_split_ws_bytes(M, N, splits, split_full));
  const int rc = rb::gemm_bf16(a.data_ptr(), lda, a_t, b.data_ptr(), ldb, b_t, out.data_ptr(), ldd, rptr, ldr,
                               M, N, K, static_cast<int>(epi), static_cast<float>(alpha), err_ptr(a), sms,
                               at::cuda::getCurrentCUDAStream(), static_cast<int>(variant),
                               splits > 1 ? ws.data_ptr() : nullptr, splits, split_full);
  TORCH_CHECK(rc == 0, "gemm_bf16 failed with code ", rc);
}


#define CHECK_BF16(t) TORCH_CHECK((t).is_cuda() && (t).scalar_type() == torch::kBFloat16 && (t).is_contiguous(), #t " must be a contiguous CUDA bf16 tensor")
#define CHECK_F32(t) TORCH_CHECK((t).is_cuda() && (t).scalar_type() == torch::kFloat32 && (t).is_contiguous(), #t " must be a contiguous CUDA fp32 tensor")
#define RB_CALL(expr, name)                                        \
  do {                                                             \
    const int rc__ = (expr);                                       \
    TORCH_CHECK(rc__ == 0, name " failed with code ", rc__);       \
  } while (0)

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

// y = rmsnorm(x) * w ; returns rstd [T]
void rmsnorm_fwd(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& y, torch::Tensor& rstd, double eps) {
  CHECK_BF16(x); CHECK_BF16(w); CHECK_BF16(y); CHECK_F32(rstd);
  const int H = x.size(-1);
  const int T = x.numel() / H;
  const c10::cuda::CUDAGuard g(x.device());
  RB_CALL(rb::rmsnorm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), T, H,
                          static_cast<float>(eps), cur_stream()), "rmsnorm_fwd");
}

void rmsnorm_bwd(const torch::Tensor& x, const torch::Tensor& w, const torch::Tensor& rstd, const torch::Tensor& dy,
                 const c10::optional<torch::Tensor>& dres, torch::Tensor& dx, torch::Tensor& dw, bool accumulate) {
  CHECK_BF16(x); CHECK_BF16(w); CHECK_F32(rstd); CHECK_BF16(dy); CHECK_BF16(dx); CHECK_F32(dw);
  const int H = x.size(-1);
  const int T = x.numel() / H;
  const void* dr = nullptr;
  if (dres.has_value()) { CHECK_BF16(*dres); dr = dres->data_ptr(); }
  const c10::cuda::CUDAGuard g(x.device());
  auto part = torch::empty({rb::rmsnorm_bwd_blocks(T), H}, x.options().dtype(torch::kFloat32));
  RB_CALL(rb::rmsnorm_bwd(x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dy.data_ptr(), dr, dx.data_ptr(),
                          dw.data_ptr<float>(), accumulate ? 1 : 0, part.data_ptr<float>(), T, H, cur_stream()),
          "rmsnorm_bwd");
}

// In-place rotary embedding on a [T, heads * D] view with row stride (elements).
void rope(torch::Tensor& t, int64_t row_stride, int64_t heads, int64_t D, const torch::Tensor& cos_t,
          const torch::Tensor& sin_t, int64_t S, int64_t T, bool inverse) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16, "rope: bf16 CUDA tensor expected");
  CHECK_F32(cos_t); CHECK_F32(sin_t);
  const c10::cuda::CUDAGuard g(t.device());
  RB_CALL(rb::rope_apply(t.data_ptr(), row_stride, heads, D, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), S, T,
                         inverse ? 1 : 0, cur_stream()), "rope");
}

void swiglu_fwd(const torch::Tensor& gu, torch::Tensor& a) {
  CHECK_BF16(gu); CHECK_BF16(a);
  const int F = a.size(-1);
  const int T = a.numel() / F;
  TORCH_CHECK(gu.numel() == 2LL * T * F, "swiglu_fwd: gu must be [T, 2F]");
  const c10::cuda::CUDAGuard g(gu.device());
  RB_CALL(rb::swiglu_fwd(gu.data_ptr(), a.data_ptr(), T, F, cur_stream()), "swiglu_fwd");
}

void swiglu_bwd(const torch::Tensor& gu, const torch::Tensor& da, torch::Tensor& dgu) {
  CHECK_BF16(gu); CHECK_BF16(da); CHECK_BF16(dgu);
  const int F = da.size(-1);
  const int T = da.numel() / F;
  const c10::cuda::CUDAGuard g(gu.device());
  RB_CALL(rb::swiglu_bwd(gu.data_ptr(), da.data_ptr(), dgu.data_ptr(), T, F, cur_stream()), "swiglu_bwd");
}

// hist [n, len] fp32, pending [n] fp32: shift the history by one and move pending into slot 0
void amax_history_push(torch::Tensor& hist, torch::Tensor& pending) {
  CHECK_F32(hist); CHECK_F32(pending);
  TORCH_CHECK(hist.dim() >= 1 && hist.numel() == pending.numel() * hist.size(-1), "amax_history_push: shapes");
  const c10::cuda::CUDAGuard g(hist.device());
  RB_CALL(rb::amax_history_push(hist.data_ptr<float>(), pending.data_ptr<float>(), pending.numel(), hist.size(-1),
                                cur_stream()), "amax_history_push");
}

void gelu_fwd(const torch::Tensor& h, torch::Tensor& a) {
  CHECK_BF16(h); CHECK_BF16(a);
  TORCH_CHECK(h.numel() == a.numel(), "gelu_fwd: sizes differ");
  const c10::cuda::CUDAGuard g(h.device());
  RB_CALL(rb::gelu_fwd(h.data_ptr(), a.data_ptr(), h.numel(), cur_stream()), "gelu_fwd");
}

void gelu_bwd(const torch::Tensor& h, const torch::Tensor& da, torch::Tensor& dh) {
  CHECK_BF16(h); CHECK_BF16(da); CHECK_BF16(dh);
  TORCH_CHECK(h.numel() == da.numel() && h.numel() == dh.numel(), "gelu_bwd: sizes differ");
  const c10::cuda::CUDAGuard g(h.device());
  RB_CALL(rb::gelu_bwd(h.data_ptr(), da.data_ptr(), dh.data_ptr(), h.numel(), cur_stream()), "gelu_bwd");
}

void embedding_fwd(const torch::Tensor& ids, const torch::Tensor& E, torch::Tensor& x) {
  TORCH_CHECK(ids.scalar_type() == torch::kInt64 && ids.is_contiguous(), "ids must be contiguous int64");
  CHECK_BF16(E); CHECK_BF16(x);
  const c10::cuda::CUDAGuard g(E.device());
  RB_CALL(rb::embedding_fwd(ids.data_ptr<int64_t>(), E.data_ptr(), x.data_ptr(), ids.numel(), E.size(1), E.size(0),
                            err_ptr(E), cur_stream()), "embedding_fwd");
}

// Deterministic dE += scatter(dx) using a stable sort of the ids.
void embedding_bwd(const torch::Tensor& ids, const torch::Tensor& dx, torch::Tensor& dE) {
  CHECK_BF16(dx); CHECK_F32(dE);
  const c10::cuda::CUDAGuard g(dx.device());
  auto flat = ids.reshape({-1});
  auto sorted = torch::sort(flat, /*stable=*/true, /*dim=*/0, /*descending=*/false);
  auto vals = std::get<0>(sorted).contiguous();
  auto order = std::get<1>(sorted).contiguous();
  RB_CALL(rb::embedding_bwd(vals.data_ptr<int64_t>(), order.data_ptr<int64_t>(), static_cast<int>(flat.numel()),
                            dx.data_ptr(), dE.data_ptr<float>(), dE.size(1), cur_stream()),
          "embedding_bwd");
}

void adam_step(torch::Tensor& p, torch::Tensor& grad, torch::Tensor& m, torch::Tensor& v,
               const c10::optional<torch::Tensor>& p_bf16, double lr, double b1, double b2, double eps, double wd,
               bool decoupled, int64_t step, double grad_scale, bool zero_grad,
               const c10::optional<torch::Tensor>& bias_corr) {
  CHECK_F32(p); CHECK_F32(grad); CHECK_F32(m); CHECK_F32(v);
  const float* bc_dev = nullptr;
  if (bias_corr.has_value()) {
    CHECK_F32((*bias_corr));
    TORCH_CHECK(bias_corr->numel() >= 2, "adam_step: bias_corr holds (1 - b1^t, sqrt(1 - b2^t))");
    bc_dev = bias_corr->data_ptr<float>();
  }
  void* pb = nullptr;
  if (p_bf16.has_value()) { CHECK_BF16(*p_bf16); TORCH_CHECK(p_bf16->numel() == p.numel()); pb = p_bf16->data_ptr(); }
  const double bc1 = 1.0 - std::pow(b1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(b2, static_cast<double>(step));
  const c10::cuda::CUDAGuard g(p.device());
  RB_CALL(rb::adam_step(p.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), pb,
                        p.numel(), lr, b1, b2, eps, wd, decoupled ? 1 : 0, static_cast<float>(bc1),
                        static_cast<float>(std::sqrt(bc2)), static_cast<float>(grad_scale), zero_grad ? 1 : 0,
                        cur_stream(), bc_dev), "adam_step");
}

// Deterministic sum of squares of a flat fp32 buffer (fixed 296-way split, fixed order).
torch::Tensor sumsq(const torch::Tensor& x) {
  CHECK_F32(x);
  const c10::cuda::CUDAGuard g(x.device());
  constexpr int kParts = 296;
  auto part = torch::empty({kParts}, x.options());
  RB_CALL(rb::sumsq_partial(x.data_ptr<float>(), x.numel(), part.data_ptr<float>(), kParts, cur_stream()), "sumsq");
  return part.sum();
}

// Fused cross-entropy: returns per-row loss (fp32); overwrites logits with dlogits when write_grad.
void cross_entropy(torch::Tensor& logits, const torch::Tensor& labels, torch::Tensor& loss,
                   const c10::optional<torch::Tensor>& lse, int64_t v0, double grad_scale, int64_t ignore_index,
                   bool write_grad) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kBFloat16 && logits.dim() == 2 &&
              logits.stride(1) == 1, "logits must be a 2-D bf16 CUDA tensor with contiguous rows");
  TORCH_CHECK(labels.scalar_type() == torch::kInt64 && labels.is_contiguous(), "labels must be int64");
  CHECK_F32(loss);
  float* lp = nullptr;
  if (lse.has_value()) { CHECK_F32(*lse); lp = lse->data_ptr<float>(); }
  const c10::cuda::CUDAGuard g(logits.device());
  RB_CALL(rb::cross_entropy_fwd_bwd(logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(),
                                    loss.data_ptr<float>(), lp, logits.size(0), logits.size(1), v0, grad_scale,
                                    ignore_index, write_grad ? 1 : 0, cur_stream()), "cross_entropy");
}

static rb::AttnArgs attn_args(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                              torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                              double scale, bool causal) {
  rb::AttnArgs a;
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr();
  a.q_stride = q.stride(0); a.k_stride = k.stride(0); a.v_stride = v.stride(0);
  a.o = o.data_ptr(); a.o_stride = o.stride(0);
  a.lse = lse.data_ptr<float>();
  a.B = B; a.S = S; a.Hq = Hq; a.Hkv = Hkv; a.scale = scale; a.causal = causal ? 1 : 0;
  return a;
}

// q/k/v/o: 2-D [B*S, heads*D] views with contiguous rows (row stride may exceed heads*D).
// impl: 0 = tcgen05 kernel when the shape allows, else mma.sync; 1 = mma.sync; 2 = tcgen05 only.
// variant (tcgen05 kernels): exponentials per 8 score columns on the FMA pipe, -1 = default.
void attention_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& o,
                   torch::Tensor& lse, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D, double scale,
                   bool causal, int64_t impl, int64_t variant) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &o})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
                "attention operands must be 2-D bf16 CUDA views with contiguous rows");
  CHECK_F32(lse);
  const c10::cuda::CUDAGuard g(q.device());
  auto a = attn_args(q, k, v, o, lse, B, S, Hq, Hkv, scale, causal);
  if (impl != 1) {
    const int rc = rb::attention_fwd_sm100(a, D, err_ptr(q), cur_stream(), static_cast<int>(variant));
    if (rc == 0) return;
    TORCH_CHECK(rc == 1 && impl == 0, "attention_fwd (tcgen05) failed with code ", rc);
  }
  RB_CALL(rb::attention_fwd_mma(a, D, cur_stream()), "attention_fwd");
}

void attention_bwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& o,
                   const torch::Tensor& dout, const torch::Tensor& lse, torch::Tensor& delta, torch::Tensor& dq,
                   torch::Tensor& dk, torch::Tensor& dv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D,
                   double scale, bool causal, int64_t impl, int64_t variant) {
  for (const torch::Tensor* t : std::initializer_list<const torch::Tensor*>{&q, &k, &v, &o, &dout, &dq, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
                "attention operands must be 2-D bf16 CUDA views with contiguous rows");
  CHECK_F32(lse); CHECK_F32(delta);
  const c10::cuda::CUDAGuard g(q.device());
  rb::AttnBwdArgs a;
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.o = o.data_ptr(); a.dout = dout.data_ptr();
  a.q_stride = q.stride(0); a.k_stride = k.stride(0); a.v_stride = v.stride(0); a.o_stride = o.stride(0);
  a.do_stride = dout.stride(0);
  a.lse = lse.data_ptr<float>(); a.delta = delta.data_ptr<float>();
  a.dq = dq.data_ptr(); a.dk = dk.data_ptr(); a.dv = dv.data_ptr();
  a.dq_stride = dq.stride(0); a.dk_stride = dk.stride(0); a.dv_stride = dv.stride(0);
  a.B = B; a.S = S; a.Hq = Hq; a.Hkv = Hkv; a.scale = scale; a.causal = causal ? 1 : 0;
  TORCH_CHECK(delta.numel() >= B * Hq * S, "delta needs B * Hq * S floats");
  if (impl != 1) {
    auto nl2 = torch::empty_like(delta);
    const int rc = rb::attention_bwd_sm100(a, D, nl2.data_ptr<float>(), err_ptr(q), cur_stream(),
                                           static_cast<int>(variant));
    if (rc == 0) return;
    TORCH_CHECK(rc == 1 && impl == 0, "attention_bwd (tcgen05) failed with code ", rc);
  }
  RB_CALL(rb::attention_bwd_mma(a, D, cur_stream()), "attention_bwd");
}


// ------------------------------------------------------------------------- symmetric peer memory
// Raw allocations of the per-generation heap; the Python side owns their lifetime.
py::tuple symm_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)) == cudaSuccess, "symm_alloc: cudaMalloc of ", bytes, " bytes failed");
  TORCH_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)) == cudaSuccess, "symm_alloc: memset failed");
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, p) == cudaSuccess, "symm_alloc: cudaIpcGetMemHandle failed");
  return py::make_tuple(reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t symm_open(const std::string& handle, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "symm_open: cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

// cuMem region of at least `bytes` on `device`, zeroed: (pointer, exported fd, mapped size).  The
// caller owns the fd (close it once every peer imported it).
py::tuple vmm_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  TORCH_CHECK(rb::vmm_available(), "vmm_alloc: the driver's cuMem entry points are unavailable");
  const long long size = rb::vmm_round(static_cast<int>(device), bytes);
  void* p = nullptr;
  int fd = -1;
  const int rc = rb::vmm_alloc(static_cast<int>(device), size, &p, &fd);
  TORCH_CHECK(rc == 0, "vmm_alloc of ", size, " bytes failed with code ", rc);
  TORCH_CHECK(cudaMemset(p, 0, static_cast<size_t>(size)) == cudaSuccess, "vmm_alloc: memset failed");
  return py::make_tuple(reinterpret_cast<int64_t>(p), static_cast<int64_t>(fd), static_cast<int64_t>(size));
}
// Map a peer's exported region (its fd, received over a Unix socket) for access from `device`.
int64_t vmm_import(int64_t fd, int64_t size, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  const int rc = rb::vmm_import(static_cast<int>(device), static_cast<int>(fd), size, &p);
  TORCH_CHECK(rc == 0, "vmm_import failed with code ", rc);
  return reinterpret_cast<int64_t>(p);
}
void vmm_free(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  const int rc = rb::vmm_free(reinterpret_cast<void*>(ptr));
  TORCH_CHECK(rc == 0, "vmm_free failed with code ", rc);
}
bool vmm_available() { return rb::vmm_available() != 0; }

void symm_free(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaFree(reinterpret_cast<void*>(ptr));
}

// Non-owning tensor view of heap memory.
torch::Tensor symm_tensor(int64_t ptr, int64_t numel, const std::string& dtype, int64_t device) {
  torch::ScalarType st;
  if (dtype == "float32") st = torch::kFloat32;
  else if (dtype == "bfloat16") st = torch::kBFloat16;
  else if (dtype == "int32") st = torch::kInt32;
  else if (dtype == "int64") st = torch::kInt64;
  else if (dtype == "uint8") st = torch::kUInt8;
  else TORCH_CHECK(false, "symm_tensor: unsupported dtype ", dtype);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {},
                          torch::TensorOptions().dtype(st).device(torch::kCUDA, device));
}

// Register an existing host mapping (e.g. an mmap'd ring file) for device access; returns the
// device address.
int64_t host_register_mapped(int64_t host_ptr, int64_t bytes) {
  void* d = nullptr;
  TORCH_CHECK(cudaHostRegister(reinterpret_cast<void*>(host_ptr), bytes, cudaHostRegisterMapped) == cudaSuccess,
              "cudaHostRegister failed");
  TORCH_CHECK(cudaHostGetDevicePointer(&d, reinterpret_cast<void*>(host_ptr), 0) == cudaSuccess,
              "cudaHostGetDevicePointer failed");
  return reinterpret_cast<int64_t>(d);
}

void host_unregister(int64_t host_ptr) { cudaHostUnregister(reinterpret_cast<void*>(host_ptr)); }

int64_t ring_record_bytes() { return rb::ring_record_bytes(); }
int64_t kernel_stamp_bytes() { return rb::kernel_stamp_bytes(); }

// Pinned, device-mapped host words (the abort word): the host writes, kernels poll.
py::tuple host_words_alloc(int64_t n) {
  void* h = nullptr;
  TORCH_CHECK(cudaHostAlloc(&h, n * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess,
              "host_words_alloc failed");
  std::memset(h, 0, n * sizeof(int));
  void* d = nullptr;
  TORCH_CHECK(cudaHostGetDevicePointer(&d, h, 0) == cudaSuccess, "cudaHostGetDevicePointer failed");
  return py::make_tuple(reinterpret_cast<int64_t>(h), reinterpret_cast<int64_t>(d));
}

void host_words_free(int64_t host_ptr) { cudaFreeHost(reinterpret_cast<void*>(host_ptr)); }

void host_word_set(int64_t host_ptr, int64_t i, int64_t value) {
  reinterpret_cast<volatile int*>(host_ptr)[i] = static_cast<int>(value);
}

int64_t host_word_get(int64_t host_ptr, int64_t i) { return reinterpret_cast<volatile int*>(host_ptr)[i]; }

int64_t symm_signal_bytes(int64_t world) { return rb::symm_signal_bytes(static_cast<int>(world)); }

// pads: int64 CUDA tensor [world] of signal-pad addresses (own pad at index rank).
void symm_barrier(const torch::Tensor& pads, int64_t rank, int64_t world, int64_t epoch, int64_t abort_dev,
                  torch::Tensor& status, double budget_s) {
  TORCH_CHECK(pads.is_cuda() && pads.scalar_type() == torch::kInt64 && pads.numel() == world, "bad pads");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32 && status.numel() >= 2, "bad status");
  const c10::cuda::CUDAGuard g(pads.device());
  RB_CALL(rb::symm_barrier(reinterpret_cast<unsigned long long* const*>(pads.data_ptr<int64_t>()),
                           static_cast<int>(rank), static_cast<int>(world), static_cast<unsigned long long>(epoch),
                           reinterpret_cast<const int*>(abort_dev), status.data_ptr<int>(), err_ptr(pads), budget_s,
                           cur_stream()), "symm_barrier");
}

void dp_step_fused(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& weight_ptrs,
                   torch::Tensor& master, torch::Tensor& m, torch::Tensor& v, int64_t shard_lo, double lr, double b1,
                   double b2, double eps, double wd, bool decoupled, int64_t step, double grad_scale,
                   int64_t abort_dev, int64_t ring_dev, int64_t ring_capacity, int64_t stamp_dev) {
  CHECK_F32(master); CHECK_F32(m); CHECK_F32(v);
  TORCH_CHECK(grad_ptrs.size() == weight_ptrs.size() && !grad_ptrs.empty(), "one grad and weight pointer per rank");
  std::vector<const float*> g(grad_ptrs.size());
  std::vector<__nv_bfloat16*> w(weight_ptrs.size());
  for (size_t i = 0; i < g.size(); ++i) {
    g[i] = reinterpret_cast<const float*>(grad_ptrs[i]);
    w[i] = reinterpret_cast<__nv_bfloat16*>(weight_ptrs[i]);
  }
  const double bc1 = 1.0 - std::pow(b1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(b2, static_cast<double>(step));
  const c10::cuda::CUDAGuard guard(master.device());
  RB_CALL(rb::dp_step_fused(g.data(), w.data(), static_cast<int>(g.size()), master.data_ptr<float>(),
                            m.data_ptr<float>(), v.data_ptr<float>(), shard_lo, master.numel(), lr, b1, b2, eps, wd,
                            decoupled ? 1 : 0, static_cast<float>(bc1), static_cast<float>(std::sqrt(bc2)),
                            static_cast<float>(grad_scale), reinterpret_cast<const int*>(abort_dev),
                            num_sms(master.get_device()), cur_stream(), reinterpret_cast<void*>(ring_dev),
                            static_cast<int>(ring_capacity), reinterpret_cast<void*>(stamp_dev)), "dp_step_fused");
}

// Slice copies (src, dst, bytes) into this rank's memory; src may be peer memory.
void symm_copy(const std::vector<int64_t>& triples, int64_t device) {
  TORCH_CHECK(triples.size() % 3 == 0, "symm_copy: triples");
  const int n = static_cast<int>(triples.size() / 3);
  long long pieces = 0;
  for (int i = 0; i < n; ++i) pieces += (triples[3 * i + 2] + (1 << 20) - 1) >> 20;
  if (pieces == 0) return;
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  auto scratch = torch::empty({pieces * rb::symm_copy_piece_bytes()},
                              torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
  RB_CALL(rb::symm_copy(reinterpret_cast<const long long*>(triples.data()), n, scratch.data_ptr(),
                        static_cast<int>(pieces), num_sms(static_cast<int>(device)), cur_stream()), "symm_copy");
}

void symm_gather(const std::vector<int64_t>& src_ptrs, int64_t dst, int64_t chunk_bytes, int64_t self,
                 int64_t device) {
  std::vector<const void*> src(src_ptrs.size());
  for (size_t c = 0; c < src_ptrs.size(); ++c) src[c] = reinterpret_cast<const void*>(src_ptrs[c]);
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  RB_CALL(rb::symm_gather(src.data(), reinterpret_cast<void*>(dst), chunk_bytes, static_cast<int>(src.size()),
                          static_cast<int>(self), num_sms(static_cast<int>(device)), cur_stream()), "symm_gather");
}

void symm_copy2d(const std::vector<int64_t>& six, int64_t device) {
  TORCH_CHECK(six.size() % 6 == 0, "symm_copy2d: sextuples");
  const int n = static_cast<int>(six.size() / 6);
  const long long pieces = rb::symm_copy2d_pieces(reinterpret_cast<const long long*>(six.data()), n);
  if (pieces == 0) return;
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  auto scratch = torch::empty({pieces * rb::symm_copy2d_piece_bytes()},
                              torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
  RB_CALL(rb::symm_copy2d(reinterpret_cast<const long long*>(six.data()), n, scratch.data_ptr(),
                          static_cast<int>(pieces), num_sms(static_cast<int>(device)), cur_stream()), "symm_copy2d");
}

// Resident piece tables: returns (device table, piece count) once; *_run launches it (no host sync).
std::tuple<torch::Tensor, int64_t> symm_copy2d_build(const std::vector<int64_t>& six, int64_t device) {
  TORCH_CHECK(six.size() % 6 == 0, "symm_copy2d_build: sextuples");
  const int n = static_cast<int>(six.size() / 6);
  const long long pieces = rb::symm_copy2d_pieces(reinterpret_cast<const long long*>(six.data()), n);
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  auto table = torch::empty({std::max<long long>(pieces, 1) * rb::symm_copy2d_piece_bytes()},
                            torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
  int count = 0;
  RB_CALL(rb::symm_copy2d_build(reinterpret_cast<const long long*>(six.data()), n, table.data_ptr(),
                                static_cast<int>(std::max<long long>(pieces, 1)), &count, cur_stream()),
          "symm_copy2d_build");
  return {table, count};
}

void symm_copy2d_run(const torch::Tensor& table, int64_t count) {
  const c10::cuda::CUDAGuard g(table.device());
  RB_CALL(rb::symm_copy2d_run(table.data_ptr(), static_cast<int>(count), num_sms(table.get_device()), cur_stream()),
          "symm_copy2d_run");
}

std::tuple<torch::Tensor, int64_t> symm_sum_build(const std::vector<int64_t>& entries, int64_t device) {
  TORCH_CHECK(entries.size() % 11 == 0, "symm_sum_build: (dst, n, nsrc, src x 8) per piece");
  const int n = static_cast<int>(entries.size() / 11);
  const long long pieces = rb::symm_sum_pieces(reinterpret_cast<const long long*>(entries.data()), n);
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  auto table = torch::empty({std::max<long long>(pieces, 1) * rb::symm_sum_piece_bytes()},
                            torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
  int count = 0;
  RB_CALL(rb::symm_sum_build(reinterpret_cast<const long long*>(entries.data()), n, table.data_ptr(),
                             static_cast<int>(std::max<long long>(pieces, 1)), &count, cur_stream()),
          "symm_sum_build");
  return {table, count};
}

void symm_sum_run(const torch::Tensor& table, int64_t count) {
  const c10::cuda::CUDAGuard g(table.device());
  RB_CALL(rb::symm_sum_run(table.data_ptr(), static_cast<int>(count), num_sms(table.get_device()), cur_stream()),
          "symm_sum_run");
}

// Tensor parallel: all-gather -> GEMM (column-parallel) and GEMM -> reduce-scatter (row-parallel).
void tp_ag_gemm(const torch::Tensor& x_full, const std::vector<int64_t>& src_ptrs, int64_t self, const torch::Tensor& w,
                bool w_t, torch::Tensor& y, torch::Tensor& ready, int64_t abort_dev) {
  CHECK_BF16(x_full); CHECK_BF16(w); CHECK_BF16(y);
  const int world = static_cast<int>(src_ptrs.size());
  const int M = x_full.size(0), K = x_full.size(1), N = w_t ? w.size(1) : w.size(0);
  TORCH_CHECK((w_t ? w.size(0) : w.size(1)) == K && y.size(0) == M && y.size(1) == N, "tp_ag_gemm: shapes");
  const int words = rb::gemm_ag_ready_words(M, K);
  TORCH_CHECK(ready.is_cuda() && ready.scalar_type() == torch::kInt32 && ready.numel() >= words,
              "tp_ag_gemm: `ready` needs ", words, " int32 words");
  std::vector<const void*> src(world);
  for (int c = 0; c < world; ++c) src[c] = reinterpret_cast<const void*>(src_ptrs[c]);
  const c10::cuda::CUDAGuard g(x_full.device());
  cudaMemsetAsync(ready.data_ptr(), 0, words * sizeof(int), cur_stream());
  RB_CALL(rb::gemm_ag_bf16(x_full.data_ptr(), src.data(), world, static_cast<int>(self), M / world, w.data_ptr(),
                           w_t, y.data_ptr(), M, N, K, ready.data_ptr<int>(), reinterpret_cast<const int*>(abort_dev),
                           err_ptr(x_full), num_sms(x_full.get_device()), cur_stream()), "tp_ag_gemm");
}

void tp_rs_gemm(const torch::Tensor& x, const torch::Tensor& w, bool w_t, const std::vector<int64_t>& recv_ptrs,
                int64_t slot) {
  CHECK_BF16(x); CHECK_BF16(w);
  const int world = static_cast<int>(recv_ptrs.size());
  std::vector<void*> recv(world);
  for (int q = 0; q < world; ++q) recv[q] = reinterpret_cast<void*>(recv_ptrs[q]);
  const int N = w_t ? w.size(1) : w.size(0);
  TORCH_CHECK((w_t ? w.size(0) : w.size(1)) == x.size(1), "tp_rs_gemm: contraction sizes differ");
  const c10::cuda::CUDAGuard g(x.device());
  RB_CALL(rb::gemm_rs_scatter_bf16(x.data_ptr(), w.data_ptr(), w_t, recv.data(), world, static_cast<int>(slot),
                                   x.size(0), N, x.size(1), err_ptr(x), num_sms(x.get_device()), cur_stream()),
          "tp_rs_gemm");
}

void tp_rs_reduce(const torch::Tensor& recv, int64_t world, torch::Tensor& out,
                  const c10::optional<torch::Tensor>& residual) {
  CHECK_BF16(recv); CHECK_BF16(out);
  TORCH_CHECK(recv.numel() >= world * out.numel(), "tp_rs_reduce: receive buffer too small");
  const c10::cuda::CUDAGuard g(out.device());
  RB_CALL(rb::rs_reduce(recv.data_ptr(), static_cast<int>(world), out.numel(), out.data_ptr(),
                        residual.has_value() ? residual->data_ptr() : nullptr, cur_stream()), "tp_rs_reduce");
}

// ------------------------------------------------------------------------- expert parallelism
static std::vector<void*> as_ptrs(const std::vector<int64_t>& v) {
  std::vector<void*> out(v.size());
  for (size_t i = 0; i < v.size(); ++i) out[i] = reinterpret_cast<void*>(v[i]);
  return out;
}

void moe_route(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& bias, int64_t k,
               torch::Tensor& logits, torch::Tensor& topi, torch::Tensor& gates) {
  CHECK_BF16(x); CHECK_BF16(w);
  const c10::cuda::CUDAGuard g(x.device());
  RB_CALL(rb::moe_route(x.data_ptr(), w.data_ptr(), bias.has_value() ? bias->data_ptr<float>() : nullptr,
                        x.size(0), x.size(1), w.size(0), k, logits.data_ptr<float>(), topi.data_ptr<int>(),
                        gates.data_ptr<float>(), cur_stream()), "moe_route");
}

void moe_positions(const torch::Tensor& topi, int64_t E, torch::Tensor& pos, torch::Tensor& counts) {
  const c10::cuda::CUDAGuard g(topi.device());
  RB_CALL(rb::moe_positions(topi.data_ptr<int>(), topi.numel(), E, pos.data_ptr<int>(), counts.data_ptr<int>(),
                            cur_stream()), "moe_positions");
}

// `routes`: int32 [E, 2 * 64 + 16] = cycle (64) | cycle rank (64) | per-cycle slots per holder (16);
// `period`: int32 [E]; `rowbase`: int64 [E, 16] (see MoeRoutes in moe.cu).
void moe_dispatch(const torch::Tensor& x, const torch::Tensor& topi, const torch::Tensor& pos, int64_t k,
                  int64_t me, const torch::Tensor& period, const torch::Tensor& routes, const torch::Tensor& rowbase,
                  const std::vector<int64_t>& recv, torch::Tensor& route_row) {
  CHECK_BF16(x);
  const int E = static_cast<int>(period.numel());
  TORCH_CHECK(routes.is_contiguous() && routes.scalar_type() == torch::kInt32 && routes.numel() == E * (2 * 64 + 16),
              "moe_dispatch: routes must be int32 [E, 144]");
  TORCH_CHECK(rowbase.is_contiguous() && rowbase.scalar_type() == torch::kInt64 && rowbase.numel() == E * 16,
              "moe_dispatch: rowbase must be int64 [E, 16]");
  const c10::cuda::CUDAGuard g(x.device());
  auto r = as_ptrs(recv);
  // split the packed table into its three [E, ...] arrays (device copies, row-major)
  auto cyc = routes.view({E, 144});
  auto cycle = cyc.narrow(1, 0, 64).contiguous();
  auto cycle_rank = cyc.narrow(1, 64, 64).contiguous();
  auto per_cycle = cyc.narrow(1, 128, 16).contiguous();
  RB_CALL(rb::moe_dispatch(x.data_ptr(), topi.data_ptr<int>(), pos.data_ptr<int>(), x.size(0), k, x.size(1),
                           static_cast<int>(r.size()), me, E, period.data_ptr<int>(), cycle.data_ptr<int>(),
                           cycle_rank.data_ptr<int>(), per_cycle.data_ptr<int>(),
                           reinterpret_cast<const long long*>(rowbase.data_ptr<int64_t>()), r.data(),
                           reinterpret_cast<long long*>(route_row.data_ptr<int64_t>()), cur_stream()),
          "moe_dispatch");
}

void moe_combine(const torch::Tensor& residual, const torch::Tensor& gates, const torch::Tensor& route_row,
                 int64_t k, const std::vector<int64_t>& ybuf, torch::Tensor& out, torch::Tensor& ycache) {
  CHECK_BF16(residual);
  const c10::cuda::CUDAGuard g(residual.device());
  auto y = as_ptrs(ybuf);
  RB_CALL(rb::moe_combine(residual.data_ptr(), gates.data_ptr<float>(),
                          reinterpret_cast<const long long*>(route_row.data_ptr<int64_t>()), residual.size(0), k,
                          residual.size(1), static_cast<int>(y.size()), y.data(), out.data_ptr(), ycache.data_ptr(),
                          cur_stream()), "moe_combine");
}

void moe_grad_push(const torch::Tensor& dout, const torch::Tensor& gates, const torch::Tensor& ycache,
                   const torch::Tensor& route_row, int64_t k, const std::vector<int64_t>& dyrecv, torch::Tensor& dgate) {
  CHECK_BF16(dout);
  const c10::cuda::CUDAGuard g(dout.device());
  auto d = as_ptrs(dyrecv);
  RB_CALL(rb::moe_grad_push(dout.data_ptr(), gates.data_ptr<float>(), ycache.data_ptr(),
                            reinterpret_cast<const long long*>(route_row.data_ptr<int64_t>()), dout.size(0), k,
                            dout.size(1), static_cast<int>(d.size()), d.data(), dgate.data_ptr<float>(), cur_stream()),
          "moe_grad_push");
}

// `residual_grad`: the gradient of the layer output, added to dx when the expert input is the
// residual stream itself; None when the experts read a normalised copy (transformer blocks).
void moe_grad_pull(const c10::optional<torch::Tensor>& residual_grad, const torch::Tensor& gates,
                   const torch::Tensor& dgate, const torch::Tensor& topi, const torch::Tensor& route_row, int64_t k,
                   int64_t E, const std::vector<int64_t>& dxbuf, torch::Tensor& dx, torch::Tensor& dlogits,
                   const c10::optional<torch::Tensor>& router_w) {
  CHECK_BF16(dx);
  if (residual_grad.has_value()) CHECK_BF16((*residual_grad));
  if (router_w.has_value()) {
    CHECK_BF16((*router_w));
    TORCH_CHECK(router_w->dim() == 2 && router_w->size(0) == E && router_w->size(1) == dx.size(1) &&
                    router_w->is_contiguous(), "moe_grad_pull: router_w must be a contiguous [E, H] tensor");
  }
  const c10::cuda::CUDAGuard g(dx.device());
  auto b = as_ptrs(dxbuf);
  RB_CALL(rb::moe_grad_pull(residual_grad.has_value() ? residual_grad->data_ptr() : nullptr, gates.data_ptr<float>(),
                            dgate.data_ptr<float>(), topi.data_ptr<int>(),
                            reinterpret_cast<const long long*>(route_row.data_ptr<int64_t>()), dx.size(0), k,
                            dx.size(1), E, static_cast<int>(b.size()), b.data(), dx.data_ptr(),
                            dlogits.data_ptr<float>(), cur_stream(),
                            router_w.has_value() ? router_w->data_ptr() : nullptr),
          "moe_grad_pull");
}

// grad [E, H] fp32 += dlogits [T, E]^T x [T, H] (bf16), two fixed-order passes (deterministic).
void moe_router_wgrad(const torch::Tensor& dlogits, const torch::Tensor& x, torch::Tensor& grad) {
  CHECK_F32(dlogits);
  CHECK_BF16(x);
  CHECK_F32(grad);
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && dlogits.dim() == 2 && dlogits.is_contiguous() &&
                  grad.is_contiguous(), "moe_router_wgrad: contiguous 2-D tensors");
  const int T = x.size(0), H = x.size(1), E = dlogits.size(1);
  TORCH_CHECK(dlogits.size(0) == T && grad.size(0) == E && grad.size(1) == H, "moe_router_wgrad: shapes");
  const c10::cuda::CUDAGuard g(x.device());
  auto ws = torch::empty({rb::moe_router_wgrad_ws_floats(T, H, E)}, grad.options());
  RB_CALL(rb::moe_router_wgrad(dlogits.data_ptr<float>(), x.data_ptr(), T, H, E, ws.data_ptr<float>(),
                               grad.data_ptr<float>(), cur_stream()),
          "moe_router_wgrad");
}

// ---------------------------------------------------------------- block-scaled fp8
static void check_fp8(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.element_size() == 1 && t.dim() == 2 && t.is_contiguous(), name,
              " must be a contiguous 2-D CUDA tensor of 1-byte elements");
}

static float* opt_f32(const c10::optional<torch::Tensor>& t, const char* name) {
  if (!t.has_value()) return nullptr;
  CHECK_F32((*t));
  return t->data_ptr<float>();
}

// RMSNorm of x [T, H] written as fp8 q [T, H] with 1x128 row-block scales s (addressing s_kb, s_row).
void rmsnorm_fp8(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& rstd, double eps,
                 int64_t fmt, const torch::Tensor& q, const torch::Tensor& s, int64_t s_kb, int64_t s_row,
                 const c10::optional<torch::Tensor>& amax) {
  CHECK_BF16(x); CHECK_BF16(w); CHECK_F32(s);
  check_fp8(q, "q");
  const int H = x.size(-1);
  const int T = x.numel() / H;
  TORCH_CHECK(q.size(0) == T && q.size(1) == H, "rmsnorm_fp8: q must be [T, H]");
  TORCH_CHECK(w.numel() == H, "rmsnorm_fp8: w must be [H]");
  TORCH_CHECK(T == 0 || (H / 128 - 1) * s_kb + static_cast<long long>(T - 1) * s_row < s.numel(), "rmsnorm_fp8: scales");
  if (rstd.has_value()) TORCH_CHECK(rstd->numel() == T, "rmsnorm_fp8: rstd must be [T]");
  const c10::cuda::CUDAGuard g(x.device());
  RB_CALL(rb::rmsnorm_fp8(x.data_ptr(), w.data_ptr(), opt_f32(rstd, "rstd"), T, H, static_cast<float>(eps),
                          static_cast<int>(fmt), q.data_ptr(), s.data_ptr<float>(), s_kb, s_row,
                          reinterpret_cast<unsigned int*>(opt_f32(amax, "amax")), cur_stream()), "rmsnorm_fp8");
}

// MLP activation of `in` ([T, F] GELU or [T, 2F] SwiGLU) written as fp8 q [T, F] with 1x128 row-block scales.
void act_fp8(const torch::Tensor& in, bool gated, int64_t fmt, const torch::Tensor& q, const torch::Tensor& s,
             int64_t s_kb, int64_t s_row, const c10::optional<torch::Tensor>& amax) {
  CHECK_BF16(in); CHECK_F32(s);
  check_fp8(q, "q");
  const int T = q.size(0), F = q.size(1);
  TORCH_CHECK(in.numel() == static_cast<long long>(T) * F * (gated ? 2 : 1), "act_fp8: input / output sizes");
  TORCH_CHECK(T == 0 || (F / 128 - 1) * s_kb + static_cast<long long>(T - 1) * s_row < s.numel(), "act_fp8: scales");
  const c10::cuda::CUDAGuard g(in.device());
  RB_CALL(rb::act_fp8(in.data_ptr(), gated ? 1 : 0, T, F, static_cast<int>(fmt), q.data_ptr(), s.data_ptr<float>(),
                      s_kb, s_row, reinterpret_cast<unsigned int*>(opt_f32(amax, "amax")), cur_stream()), "act_fp8");
}

// Quantise bf16 x [R, C]; outputs are optional (rowwise q [R, C], colwise q [C, R]).
void fp8_quantize(const torch::Tensor& x, int64_t fmt, bool two_d, const c10::optional<torch::Tensor>& q_row,
                  const c10::optional<torch::Tensor>& s_row, const c10::optional<torch::Tensor>& q_col,
                  const c10::optional<torch::Tensor>& s_col, const c10::optional<torch::Tensor>& amax,
                  bool row_major, int64_t act) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2, "x must be a 2-D CUDA bf16 tensor");
  TORCH_CHECK(act >= 0 && act <= 2, "fp8_quantize: act is 0 (none), 1 (gelu) or 2 (swiglu)");
  const long long ldx = ld_of(x, "x");
  const int R = x.size(0), C = act == 2 ? x.size(1) / 2 : x.size(1);
  const long long nr = (R / 128), nc = (C / 128);  // R need not be a multiple of 128 for rowwise-only output
  if (q_row.has_value()) {
    check_fp8(*q_row, "q_row");
    TORCH_CHECK(q_row->size(0) == R && q_row->size(1) == C, "q_row must be [R, C]");
  }
  if (q_col.has_value()) {
    check_fp8(*q_col, "q_col");
    TORCH_CHECK(q_col->size(0) == C && q_col->size(1) == R, "q_col must be [C, R]");
  }
  if (s_row.has_value()) TORCH_CHECK(s_row->numel() == (two_d ? nr * nc : static_cast<long long>(R) * nc), "bad s_row size");
  if (s_col.has_value()) TORCH_CHECK(s_col->numel() == nr * C, "bad s_col size");
  if (amax.has_value()) TORCH_CHECK(amax->numel() >= 1, "amax needs one element");
  const c10::cuda::CUDAGuard g(x.device());
  RB_CALL(rb::fp8_quantize(x.data_ptr(), ldx, R, C, static_cast<int>(fmt), two_d ? 1 : 0,
                           q_row.has_value() ? q_row->data_ptr() : nullptr, opt_f32(s_row, "s_row"),
                           q_col.has_value() ? q_col->data_ptr() : nullptr, opt_f32(s_col, "s_col"),
                           reinterpret_cast<unsigned int*>(opt_f32(amax, "amax")), cur_stream(), row_major ? 1 : 0,
                           static_cast<int>(act)),
          "fp8_quantize");
}

static void check_scale(const torch::Tensor& s, int64_t kb, int64_t row, int64_t shift, int rows, int K,
                        const char* name) {
  CHECK_F32(s);
  TORCH_CHECK(kb >= 0 && row >= 0 && (shift == 0 || shift == 7), name, ": bad scale addressing");
  TORCH_CHECK(rows > 0 && K >= 128 && K % 128 == 0, name, ": needs rows > 0 and K a positive multiple of 128");
  const long long last = (static_cast<long long>(K / 128) - 1) * kb + static_cast<long long>((rows - 1) >> shift) * row;
  TORCH_CHECK(last >= 0 && last < s.numel(), name, ": scale tensor too small for its addressing");
}

// out[M, N] (+)= alpha * sum_kb sa(m, kb) sb(n, kb) (a[m, kb] . b[n, kb])
void gemm_fp8(const torch::Tensor& a, int64_t a_fmt, const torch::Tensor& sa, int64_t sa_kb, int64_t sa_row,
              int64_t sa_shift, const torch::Tensor& b, int64_t b_fmt, const torch::Tensor& sb, int64_t sb_kb,
              int64_t sb_row, int64_t sb_shift, const c10::optional<torch::Tensor>& out, int64_t epi, double alpha,
              const c10::optional<torch::Tensor>& residual, const std::vector<int64_t>& rs_ptrs, int64_t rs_slot,
              int64_t variant) {
  check_fp8(a, "a");
  TORCH_CHECK(variant >= 0 && variant <= 3, "gemm_fp8: variant is 0 (auto), 1 (register promotion), 2 (single-CTA tensor-core scaling) or 3 (CTA pair)");
  check_fp8(b, "b");
  // Every shape rule of the kernel is checked here, before any pointer or tensor map is formed.
  TORCH_CHECK(a.size(0) > 0 && a.size(1) > 0 && b.size(0) > 0 && a.size(0) % 128 == 0 && a.size(1) % 128 == 0 &&
                  b.size(0) % 128 == 0,
              "gemm_fp8: M, N and K must be positive multiples of 128");
  TORCH_CHECK(a_fmt == 0 || a_fmt == 1, "gemm_fp8: a_fmt is 0 (E4M3) or 1 (E5M2)");
  TORCH_CHECK(b_fmt == 0 || b_fmt == 1, "gemm_fp8: b_fmt is 0 (E4M3) or 1 (E5M2)");
  TORCH_CHECK(epi >= 0 && epi <= 4, "gemm_fp8: epi is 0..4");
  TORCH_CHECK(a.device() == b.device(), "gemm_fp8: a and b on different devices");
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K, "gemm_fp8: contraction sizes differ");
  void* dptr = nullptr;
  long long ldd = 0;
  std::vector<void*> dst;
  if (epi == 4) {  // scatter into receive slots (peer memory); no local output
    TORCH_CHECK(!rs_ptrs.empty(), "gemm_fp8: the scatter epilogue needs receive pointers");
    for (auto p : rs_ptrs) dst.push_back(reinterpret_cast<void*>(p));
  } else {
    TORCH_CHECK(out.has_value(), "gemm_fp8: out is required");
    const auto& o = *out;
    TORCH_CHECK(o.is_cuda() && o.dim() == 2 && o.size(0) == M && o.size(1) == N, "gemm_fp8: out must be [M, N]");
    TORCH_CHECK(o.scalar_type() == ((epi == 0 || epi == 3) ? torch::kBFloat16 : torch::kFloat32), "gemm_fp8: out dtype");
    dptr = o.data_ptr();
    ldd = ld_of(o, "out");
  }
  const void* rptr = nullptr;
  long long ldr = 0;
  if (epi == 3) {
    TORCH_CHECK(residual.has_value(), "gemm_fp8: the residual epilogue needs a residual");
    const auto& r = *residual;
    TORCH_CHECK(r.is_cuda() && r.scalar_type() == torch::kBFloat16 && r.size(0) == M && r.size(1) == N, "bad residual");
    rptr = r.data_ptr();
    ldr = ld_of(r, "residual");
  }
  check_scale(sa, sa_kb, sa_row, sa_shift, M, K, "sa");
  check_scale(sb, sb_kb, sb_row, sb_shift, N, K, "sb");
  TORCH_CHECK(variant != 3 || M % 256 == 0, "gemm_fp8: the CTA-pair kernel (variant 3) needs M a multiple of 256");
  if (variant == 1 && sb_shift == 0)
    TORCH_CHECK(sb_row == 1 && sb_kb % 4 == 0 && reinterpret_cast<uintptr_t>(sb.data_ptr()) % 16 == 0,
                "gemm_fp8: per-column B scales need unit row stride, K-block stride a multiple of 4, 16-byte base");
  const c10::cuda::CUDAGuard g(a.device());
  torch::Tensor sf_ws;  // packed scale words of the block-scaled path (stream-ordered, from the caching allocator)
  if (variant != 1) sf_ws = torch::empty({rb::gemm_fp8_sf_bytes(M, N, K)}, a.options().dtype(torch::kUInt8));
  // (variant 0 may still pick the register-promotion kernel for a small product; it then leaves
  // the workspace unused)
  RB_CALL(rb::gemm_fp8(a.data_ptr(), static_cast<int>(a_fmt), b.data_ptr(), static_cast<int>(b_fmt),
                       sa.data_ptr<float>(), sa_kb, sa_row, static_cast<int>(sa_shift), sb.data_ptr<float>(), sb_kb,
                       sb_row, static_cast<int>(sb_shift), dptr, ldd, M, N, K, static_cast<int>(epi),
                       static_cast<float>(alpha), err_ptr(a), num_sms(a.get_device()), cur_stream(), rptr, ldr,
                       dst.empty() ? nullptr : dst.data(), static_cast<int>(dst.size()), static_cast<int>(rs_slot),
                       static_cast<int>(variant), sf_ws.defined() ? sf_ws.data_ptr() : nullptr),
          "gemm_fp8");
}

torch::Tensor error_state(int64_t device) { return error_word(static_cast<int>(device)); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of resihp_megatron_b200";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("a_t"), py::arg("b"), py::arg("b_t"),
        py::arg("out"), py::arg("epi"), py::arg("alpha"), py::arg("residual") = py::none(),
        py::arg("variant") = 0);
  m.def("error_state", &error_state, "per-device kernel error words");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("gelu_fwd", &gelu_fwd);
  m.def("amax_history_push", &amax_history_push);
  m.def("gelu_bwd", &gelu_bwd);
  m.def("fp8_quantize", &fp8_quantize, "block-scaled fp8 quantisation", py::arg("x"), py::arg("fmt"),
        py::arg("two_d"), py::arg("q_row"), py::arg("s_row"), py::arg("q_col"), py::arg("s_col"), py::arg("amax"),
        py::arg("row_major") = false, py::arg("act") = 0);
  m.def("act_fp8", &act_fp8, "MLP activation written as block-scaled fp8", py::arg("input"), py::arg("gated"),
        py::arg("fmt"), py::arg("q"), py::arg("s"), py::arg("s_kb"), py::arg("s_row"), py::arg("amax"));
  m.def("rmsnorm_fp8", &rmsnorm_fp8, "RMSNorm written as block-scaled fp8", py::arg("x"), py::arg("w"),
        py::arg("rstd"), py::arg("eps"), py::arg("fmt"), py::arg("q"), py::arg("s"), py::arg("s_kb"), py::arg("s_row"),
        py::arg("amax"));
  m.def("gemm_fp8", &gemm_fp8, "tcgen05 block-scaled fp8 GEMM", py::arg("a"), py::arg("a_fmt"), py::arg("sa"),
        py::arg("sa_kb"), py::arg("sa_row"), py::arg("sa_shift"), py::arg("b"), py::arg("b_fmt"), py::arg("sb"),
        py::arg("sb_kb"), py::arg("sb_row"), py::arg("sb_shift"), py::arg("out"), py::arg("epi"), py::arg("alpha"),
        py::arg("residual") = py::none(), py::arg("rs_ptrs") = std::vector<int64_t>{}, py::arg("rs_slot") = 0,
        py::arg("variant") = 0);
  m.def("adam_step", &adam_step);
  m.def("sumsq", &sumsq);
  m.def("cross_entropy", &cross_entropy);
  m.def("attention_fwd", &attention_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("B"), py::arg("S"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("scale"), py::arg("causal"),
        py::arg("impl") = 0, py::arg("variant") = -1);
  m.def("tp_ag_ready_words", [](int64_t M, int64_t K) { return rb::gemm_ag_ready_words(M, K); });
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("vmm_alloc", &vmm_alloc);
  m.def("vmm_import", &vmm_import);
  m.def("vmm_free", &vmm_free);
  m.def("vmm_available", &vmm_available);
  m.def("symm_tensor", &symm_tensor);
  m.def("host_words_alloc", &host_words_alloc);
  m.def("host_words_free", &host_words_free);
  m.def("host_word_set", &host_word_set);
  m.def("host_word_get", &host_word_get);
  m.def("symm_signal_bytes", &symm_signal_bytes);
  m.def("symm_barrier", &symm_barrier);
  m.def("dp_step_fused", &dp_step_fused);
  m.def("symm_copy", &symm_copy);
  m.def("symm_gather", &symm_gather);
  m.def("symm_copy2d", &symm_copy2d);
  m.def("host_register_mapped", &host_register_mapped);
  m.def("host_unregister", &host_unregister);
  m.def("ring_record_bytes", &ring_record_bytes);
  m.def("kernel_stamp_bytes", &kernel_stamp_bytes);
  m.def("tp_ag_gemm", &tp_ag_gemm);
  m.def("moe_route", &moe_route);
  m.def("moe_positions", &moe_positions);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_combine", &moe_combine);
  m.def("moe_grad_push", &moe_grad_push);
  m.def("moe_grad_pull", &moe_grad_pull, "expert-parallel gradient pull (+ the router path)", py::arg("residual_grad"),
        py::arg("gates"), py::arg("dgate"), py::arg("topi"), py::arg("route_row"), py::arg("k"), py::arg("E"),
        py::arg("dxbuf"), py::arg("dx"), py::arg("dlogits"), py::arg("router_w") = py::none());
  m.def("moe_router_wgrad", &moe_router_wgrad, "router weight gradient, deterministic");
  m.def("tp_rs_gemm", &tp_rs_gemm);
  m.def("symm_copy2d_build", &symm_copy2d_build);
  m.def("symm_copy2d_run", &symm_copy2d_run);
  m.def("symm_sum_build", &symm_sum_build);
  m.def("symm_sum_run", &symm_sum_run);
  m.def("tp_rs_reduce", &tp_rs_reduce, py::arg("recv"), py::arg("world"), py::arg("out"),
        py::arg("residual") = py::none());
  m.def("attention_bwd", &attention_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dout"),
        py::arg("lse"), py::arg("delta"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("B"), py::arg("S"),
        py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("scale"), py::arg("causal"), py::arg("impl") = 0,
        py::arg("variant") = -1);
}
