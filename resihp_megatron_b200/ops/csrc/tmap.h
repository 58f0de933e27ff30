// TMA tensor-map construction shared by the tcgen05 kernels (implemented in gemm_sm100.cu).
#pragma once

#include <cuda.h>

#include <cstdint>

namespace rb {

// 2-D tensor map with 128-byte swizzle over a row-major matrix of `elem_bytes`-byte elements:
// `inner` contiguous elements per row, `outer` rows, rows `row_stride_elems` elements apart,
// boxes of `box_inner` x `box_outer` elements.  Returns 0 or a CUresult.
int make_tmap_2d_sw128(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes, const void* ptr, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer);

// The same without swizzle (rows of the box land contiguously in shared memory).
int make_tmap_2d_plain(CUtensorMap* tm, CUtensorMapDataType dtype, int elem_bytes, const void* ptr, uint64_t inner,
                       uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer);

}  // namespace rb
