// tensormap.cpp — cuTensorMapEncodeTiled through the runtime's driver
// entry-point lookup.
#include "tensormap.h"

#include <mutex>

namespace infernt {

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;
std::once_flag g_once;
cudaError_t g_lookup = cudaSuccess;
}  // namespace

cudaError_t encode_weight_map(CUtensorMap* map, const void* W, int rows, int K, int elem_bytes, int box_rows) {
    std::call_once(g_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        g_lookup = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (g_lookup == cudaSuccess && q != cudaDriverEntryPointSuccess) g_lookup = cudaErrorNotSupported;
        g_encode = reinterpret_cast<EncodeFn>(fn);
    });
    if (g_lookup != cudaSuccess || !g_encode) return g_lookup != cudaSuccess ? g_lookup : cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * (cuuint64_t)elem_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)kBoxCols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = g_encode(map, dt, 2, const_cast<void*>(W), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace infernt
