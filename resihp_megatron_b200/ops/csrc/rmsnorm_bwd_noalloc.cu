// Allocation-free RMSNorm backward: the same kernels as rb::rmsnorm_bwd, with the per-CTA
// partial weight-gradient buffer taken from a file-scope __device__ array instead of an
// allocator.  See rmsnorm_bwd_noalloc.h for who needs this and for the call contract.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"
#include "rmsnorm_bwd_noalloc.h"

namespace {

// One copy per device that loads this library, alive until process exit.  In host code this
// name is only a host-side stand-in; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_rmsnorm_scratch[RB_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};
void* g_scratch_ctx[kMaxDevices] = {};  // the context the cached address belongs to

// The current driver context, through the runtime's driver entry point (no link to libcuda).
void* current_context() {
  using GetCurrentFn = int (*)(void**);
  static GetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<GetCurrentFn>(f);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of the scratch array on the current device.  Looked up once per device and
// context: after a cudaDeviceReset (or any re-creation of the device's primary context) the
// context handle changes, and the address is looked up again instead of reusing a stale one.
int scratch_on_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return RB_NOALLOC_ERR_SYMBOL;
  std::lock_guard<std::mutex> lock(g_mu);
  void* ctx = current_context();
  if (g_scratch_ptr[dev] == nullptr || ctx == nullptr || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rmsnorm_scratch);
    if (e != cudaSuccess || p == nullptr) return RB_NOALLOC_ERR_SYMBOL;
    g_scratch_ptr[dev] = static_cast<float*>(p);
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int rb_rmsnorm_bwd_noalloc(const void* x, const void* w, const float* rstd, const void* dy,
                                      const void* dres, void* dx, float* dw, int accumulate, int T, int H,
                                      cudaStream_t stream) {
  if (T <= 0 || H <= 0 || H % 8 != 0 || H > 8192) return RB_NOALLOC_ERR_BAD_SHAPE;
  const long long need = static_cast<long long>(rb::rmsnorm_bwd_blocks(T)) * H;
  if (need > RB_NOALLOC_SCRATCH_FLOATS) return RB_NOALLOC_ERR_TOO_LARGE;
  float* scratch = nullptr;
  if (int rc = scratch_on_current_device(&scratch)) return rc;
  return rb::rmsnorm_bwd(x, w, rstd, dy, dres, dx, dw, accumulate, scratch, T, H, stream);
}

extern "C" long long rb_rmsnorm_bwd_noalloc_capacity(void) { return RB_NOALLOC_SCRATCH_FLOATS; }
