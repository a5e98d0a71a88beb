// Definitions of the shared host helpers (host_util.cuh).
#include "host_util.cuh"

#include <cstdarg>
#include <cstdio>

namespace cgdr {
namespace host {

thread_local char g_err[512] = "";

cgdrStatus fail(cgdrStatus st, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return st;
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

}  // namespace

cgdrStatus make_map(CUtensorMap* map, void* base, int rank, const int64_t* size, const int64_t* stride,
                    const uint32_t* box, const char* name, int swizzle_bytes)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(CGDR_STATUS_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t gdim[5], gstride[4];
    cuuint32_t bdim[5], estride[5];
    for (int i = 0; i < rank; ++i) {
        gdim[i] = static_cast<cuuint64_t>(size[i] > 0 ? size[i] : 1);
        bdim[i] = box[i];
        estride[i] = 1;
    }
    for (int i = 1; i < rank; ++i) gstride[i - 1] = static_cast<cuuint64_t>(stride[i]) * 2;
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base, gdim, gstride, bdim, estride,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle_bytes == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CGDR_STATUS_CUDA_ERROR, "cuTensorMapEncodeTiled(%s) failed: %d", name, (int)r);
    return CGDR_STATUS_SUCCESS;
}

}  // namespace host
}  // namespace cgdr
