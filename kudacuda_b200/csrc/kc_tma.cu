// kc_tma.cu -- tensor-map encoding through the driver entry point.
#include "kc_tma.h"

#include <atomic>

namespace kc {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static std::atomic<EncodeTiledFn> cached{nullptr};
    EncodeTiledFn f = cached.load(std::memory_order_acquire);
    if (f != nullptr) return f;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
        return nullptr;
    f = reinterpret_cast<EncodeTiledFn>(p);
    cached.store(f, std::memory_order_release);
    return f;
}

}  // namespace

cudaError_t encode_tmap_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                           uint64_t rows, uint64_t row_stride, uint32_t box_inner, uint32_t box_rows,
                           CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promotion) {
    EncodeTiledFn f = encode_fn();
    if (f == nullptr) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = f(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle, promotion, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace kc
