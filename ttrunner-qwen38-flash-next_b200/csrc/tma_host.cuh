// Host side of 2-D TMA tensor copies: cuTensorMapEncodeTiled obtained through
// the runtime's driver entry point (no link against the driver library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace qmoe {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiledFn) nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// A row-major 2-D tensor of `rows` rows, `inner` elements each (row pitch
// `row_bytes`, a multiple of 16; base 16-byte aligned), copied in boxes of
// box_inner x box_rows elements (optionally 128-byte swizzled: box rows of
// 128 bytes, 16-byte chunk j of row r landing at chunk j ^ (r & 7)); reads
// past the edges return zero.
inline cudaError_t encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, unsigned long long inner,
                             unsigned long long rows, unsigned long long row_bytes, unsigned box_inner,
                             unsigned box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace qmoe
