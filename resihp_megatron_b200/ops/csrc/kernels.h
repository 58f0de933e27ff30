// Host-side entry points of the sm_100a kernels (implemented in the *.cu files of this
// directory).  All functions return 0 on success; negative values flag bad arguments and
// positive values are CUDA error codes.
#pragma once

#include <cuda_runtime.h>

namespace rb {

int gemm_bf16(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* D,
              long long ldd, const void* R, long long ldr, int M, int N, int K, int epi, float alpha,
              int* err, int num_sms, cudaStream_t stream);

}  // namespace rb
