// kc_tma.h -- TMA tensor-map encoding (host) for the bulk-tensor kernels.
//
// The driver function cuTensorMapEncodeTiled is resolved at run time through
// cudaGetDriverEntryPoint, so the library keeps no link-time dependency on
// libcuda.  Encoding is a pure host computation: it is safe during CUDA graph
// capture and the maps travel to the kernel by value as __grid_constant__
// parameters.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kc {

// 2D row-major tensor [rows][inner] of `elem_bytes`-sized elements starting at
// `base`; rows are `row_stride` bytes apart.  Box = box_rows x box_inner
// elements.  Returns cudaErrorInvalidValue when the driver rejects the map
// (alignment, strides) or the entry point is missing.
cudaError_t encode_tmap_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                           uint64_t rows, uint64_t row_stride, uint32_t box_inner, uint32_t box_rows,
                           CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promotion);

}  // namespace kc
