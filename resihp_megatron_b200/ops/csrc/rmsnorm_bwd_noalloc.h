// RMSNorm backward for callers that cannot allocate device memory.
//
// This entry point has no counterpart in the reference framework; it exists for users of
// this library, not for parity.
//
// Who needs it: code that calls this library from inside another program's process without
// access to that program's allocator -- a C or Fortran host application, a plugin loaded
// into an inference or training server, a tool that runs next to a job on a GPU whose
// memory is fully reserved.  For them cudaMalloc is off limits: it can fail when the host
// program has reserved all device memory, it implicitly synchronises the device (stalling
// the host program's streams), and memory it returns escapes the host program's accounting.
// The regular entry point (`rb::rmsnorm_bwd`, used through the Python bindings) gets its
// scratch buffer from the PyTorch caching allocator, which these callers do not have.
//
// Contract of rb_rmsnorm_bwd_noalloc:
//  * Allocates nothing: no cudaMalloc / cudaFree / allocating library call.  Its scratch is a
//    file-scope __device__ array of RB_NOALLOC_SCRATCH_FLOATS floats (2 MiB) that every GPU
//    which loads this library holds until the process exits.
//  * Scratch needed: ceil(T / 32) * H floats.  Calls that need more return
//    RB_NOALLOC_ERR_TOO_LARGE and launch nothing (e.g. H = 4096 allows T <= 4096 rows).
//  * The first call on a device (with that device current) looks up the array's device
//    address with cudaGetSymbolAddress and caches it with the device's current context; make
//    that first call before any stream capture on that device.  If the context changes (a
//    cudaDeviceReset, or the primary context released and created again), the next call looks
//    the address up again, so that call too should come outside a stream capture.
//  * Every call on a device shares the one array, and the array keeps the previous call's
//    contents.  The kernels overwrite every scratch element they read, so nothing needs
//    clearing between calls.  Calls that overlap on the GPU (different streams without
//    ordering between them) race on the array: serialise them.
//  * Inputs and outputs are caller-owned device pointers (bf16 x, w, dy, optional dres, dx;
//    fp32 rstd and dw); `stream` may be 0.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RB_NOALLOC_SCRATCH_FLOATS (512 * 1024)

#define RB_NOALLOC_OK 0
#define RB_NOALLOC_ERR_TOO_LARGE -2      /* ceil(T/32) * H > RB_NOALLOC_SCRATCH_FLOATS */
#define RB_NOALLOC_ERR_BAD_SHAPE -3      /* T <= 0, H <= 0, H % 8 != 0 or H > 8192 */
#define RB_NOALLOC_ERR_SYMBOL -4         /* cudaGetSymbolAddress failed on this device */

// dx = d(rmsnorm(x) * w)/dx . dy (+ dres when non-null); dw = (accumulate ? dw : 0) + sum_rows dy * xhat.
// Returns 0, one of the RB_NOALLOC_ERR_* codes, or a positive cudaError_t.
int rb_rmsnorm_bwd_noalloc(const void* x, const void* w, const float* rstd, const void* dy, const void* dres,
                           void* dx, float* dw, int accumulate, int T, int H, cudaStream_t stream);

// Largest number of scratch floats a call may need (RB_NOALLOC_SCRATCH_FLOATS).
long long rb_rmsnorm_bwd_noalloc_capacity(void);

#ifdef __cplusplus
}
#endif
