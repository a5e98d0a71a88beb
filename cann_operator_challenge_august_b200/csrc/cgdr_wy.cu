// Host side of include/cgdr_wy.h: validation, plan, tensor maps and the
// launch of the WY kernel.  No device memory is allocated here.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "../../include/cgdr_wy.h"
#include "host_stages.cuh"
#include "host_util.cuh"
#include "kernel_wy.cuh"

using namespace cgdr;
using namespace cgdr::host;

struct cgdrWyExecutor {
    uint32_t magic;
    WyParams p;
    cgdrTensor tk, tv;
    int64_t grid;
};

namespace {

constexpr uint32_t kMagicWy = 0xC6D2A7B1u;
constexpr uint64_t kHeader = 256;
constexpr int kStagesWy = 3;

int64_t sm_count_wy()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        n > 0)
        return n;
    cudaGetLastError();
    return 148;
}

// 16-byte aligned base and rows (the kernel writes w and u with 16-byte stores)
bool rows16(const cgdrTensor* t)
{
    if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return false;
    for (int i = 0; i < t->ndim - 1; ++i)
        if ((t->strides[i] * 2) % 16 != 0) return false;
    return true;
}

cgdrStatus build_wy(const cgdrTensor* k, const cgdrTensor* v, const cgdrTensor* beta, const cgdrTensor* g,
                    const cgdrTensor* cu, const cgdrTensor* ci, int64_t chunk_size, const cgdrTensor* w,
                    const cgdrTensor* u, const cgdrTensor* gc, const cgdrWyOptions* opt, uint64_t* ws_size,
                    cgdrWyExecutor** out)
{
    if (!ws_size || !out) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace_size and executor must not be NULL");
    *out = nullptr;
    if (!present(k) || !present(v) || !present(beta) || !present(w) || !present(u))
        return fail(CGDR_STATUS_NULL_ARGUMENT, "k, v, beta, w and u are required");
    const bool has_cu = present(cu), has_ci = present(ci);
    if (has_cu != has_ci)
        return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens and chunk_indices must be both present or both absent");
    cgdrStatus st;
    if ((st = check_rank(k, 4, "k")) || (st = check_rank(v, 4, "v")) || (st = check_rank(beta, 3, "beta")) ||
        (st = check_rank(w, 4, "w")) || (st = check_rank(u, 4, "u")))
        return st;
    if (present(g) && (st = check_rank(g, 3, "g"))) return st;
    if (present(gc) && (st = check_rank(gc, 3, "g_cum"))) return st;
    if (has_cu && ((st = check_rank(cu, 1, "cu_seqlens")) || (st = check_rank(ci, 2, "chunk_indices")))) return st;
    for (const cgdrTensor* t : {k, v, beta, w, u})
        if (t->dtype != CGDR_DT_BF16) return fail(CGDR_STATUS_BAD_DTYPE, "k, v, beta, w and u must be bfloat16");
    if ((present(g) && g->dtype != CGDR_DT_FLOAT32) || (present(gc) && gc->dtype != CGDR_DT_FLOAT32))
        return fail(CGDR_STATUS_BAD_DTYPE, "g and g_cum must be float32");
    if (has_cu && (cu->dtype != CGDR_DT_INT64 || ci->dtype != CGDR_DT_INT64))
        return fail(CGDR_STATUS_BAD_DTYPE, "cu_seqlens and chunk_indices must be int64");
    if (chunk_size != kChunk)
        return fail(CGDR_STATUS_BAD_CHUNK_SIZE, "chunk_size must be 64, got %lld", static_cast<long long>(chunk_size));

    const int64_t B = k->shape[0], T = k->shape[1], HK = k->shape[2], K = k->shape[3];
    const int64_t H = v->shape[2], V = v->shape[3];
    if (B <= 0 || T < 0 || HK <= 0 || K <= 0 || H <= 0 || V <= 0)
        return fail(CGDR_STATUS_BAD_SHAPE, "dimensions must be positive");
    if (v->shape[0] != B || v->shape[1] != T) return fail(CGDR_STATUS_BAD_SHAPE, "v must have shape [B, T, HV, V]");
    if (H % HK != 0) return fail(CGDR_STATUS_BAD_SHAPE, "HV must be divisible by HK");
    if (!shape_is(beta, {B, T, H})) return fail(CGDR_STATUS_BAD_SHAPE, "beta must have shape [B, T, HV]");
    if (present(g) && !shape_is(g, {B, T, H})) return fail(CGDR_STATUS_BAD_SHAPE, "g must have shape [B, T, HV]");
    if (present(gc) && !shape_is(gc, {B, T, H})) return fail(CGDR_STATUS_BAD_SHAPE, "g_cum must have shape [B, T, HV]");
    if (!shape_is(w, {B, T, H, K})) return fail(CGDR_STATUS_BAD_SHAPE, "w must have shape [B, T, HV, K]");
    if (!shape_is(u, {B, T, H, V})) return fail(CGDR_STATUS_BAD_SHAPE, "u must have shape [B, T, HV, V]");
    int64_t N = B, NT = (T + kChunk - 1) / kChunk, rows = B * NT;
    if (has_cu) {
        if (B != 1) return fail(CGDR_STATUS_BAD_VARLEN, "variable-length input needs B == 1");
        if (cu->shape[0] < 2) return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens needs at least two entries");
        if (ci->shape[1] != 2) return fail(CGDR_STATUS_BAD_VARLEN, "chunk_indices must have shape [NT, 2]");
        if (cu->shape[0] > 1 && cu->strides[0] != 1) return fail(CGDR_STATUS_BAD_STRIDE, "cu_seqlens must be contiguous");
        if (ci->strides[1] != 1 || ci->strides[0] != 2)
            return fail(CGDR_STATUS_BAD_STRIDE, "chunk_indices must be contiguous");
        N = cu->shape[0] - 1;
        NT = ci->shape[0];
        rows = NT;
        const int64_t nt_min = (T + kChunk - 1) / kChunk;
        if (NT < nt_min || NT > nt_min + N - 1)
            return fail(CGDR_STATUS_BAD_VARLEN, "NT=%lld is impossible for T=%lld and N=%lld",
                        static_cast<long long>(NT), static_cast<long long>(T), static_cast<long long>(N));
    }
    for (const cgdrTensor* t : {k, v, w, u})
        if ((st = check_inner_contiguous(t, "k/v/w/u"))) return st;
    for (const cgdrTensor* t : {beta, g, gc})
        if (present(t))
            for (int i = 0; i < t->ndim; ++i)
                if (t->strides[i] < 0) return fail(CGDR_STATUS_BAD_STRIDE, "negative stride");
    if (!(K == 64 || K == 128) || !(V == 64 || V == 128))
        return fail(CGDR_STATUS_UNSUPPORTED, "the WY kernel is built for K and V in {64, 128}");
    if (!tma_aligned(k) || !tma_aligned(v) || !rows16(w) || !rows16(u))
        return fail(CGDR_STATUS_BAD_STRIDE, "k, v, w and u need 16-byte aligned bases and strides");
    if (T >= (int64_t(1) << 31)) return fail(CGDR_STATUS_UNSUPPORTED, "T must fit in 31 bits");

    cgdrWyExecutor* ex = new (std::nothrow) cgdrWyExecutor();
    if (!ex) return fail(CGDR_STATUS_UNSUPPORTED, "out of host memory");
    ex->magic = kMagicWy;
    WyParams& p = ex->p;
    memset(&p, 0, sizeof(p));
    p.beta = static_cast<const __nv_bfloat16*>(beta->data);
    p.g = present(g) ? static_cast<const float*>(g->data) : nullptr;
    p.w = static_cast<__nv_bfloat16*>(w->data);
    p.u = static_cast<__nv_bfloat16*>(u->data);
    p.g_cum = present(gc) ? static_cast<float*>(gc->data) : nullptr;
    p.cu_seqlens = has_cu ? static_cast<const int64_t*>(cu->data) : nullptr;
    p.chunk_indices = has_cu ? static_cast<const int64_t*>(ci->data) : nullptr;
    p.B = B; p.T = T; p.H = H; p.HK = HK; p.K = K; p.V = V; p.N = N; p.NT = NT;
    p.nt_per_seq = (T + kChunk - 1) / kChunk;
    p.n_tiles = rows * H;
    p.b_sb = beta->strides[0]; p.b_st = beta->strides[1]; p.b_sh = beta->strides[2];
    if (present(g)) { p.g_sb = g->strides[0]; p.g_st = g->strides[1]; p.g_sh = g->strides[2]; }
    if (present(gc)) { p.c_sb = gc->strides[0]; p.c_st = gc->strides[1]; p.c_sh = gc->strides[2]; }
    p.w_sb = w->strides[0]; p.w_st = w->strides[1]; p.w_sh = w->strides[2];
    p.u_sb = u->strides[0]; p.u_st = u->strides[1]; p.u_sh = u->strides[2];
    p.varlen = has_cu ? 1 : 0;
    const int32_t tmo = opt && opt->wait_timeout_ms > 0 ? opt->wait_timeout_ms : 2000;
    p.timeout_ns = static_cast<uint64_t>(tmo) * 1000000ull;
    ex->tk = *k;
    ex->tv = *v;
    const int64_t sms = sm_count_wy();
    ex->grid = p.n_tiles < sms ? p.n_tiles : sms;
    *ws_size = kHeader;
    *out = ex;
    g_err[0] = '\0';
    return CGDR_STATUS_SUCCESS;
}

template <int K_, int V_>
cudaError_t launch_wy(const WyArgs& args, int64_t grid, cudaStream_t stream)
{
    using Cfg = WyConfig<K_, V_, kStagesWy>;
    auto kern = wy_tc_kernel<K_, V_, kStagesWy>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(grid), Cfg::kThreads, Cfg::kSmemBytes, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace

extern "C" {

cgdrStatus cgdrChunkGatedDeltaRuleWYGetWorkspaceSize(const cgdrTensor* k, const cgdrTensor* v, const cgdrTensor* beta,
                                                     const cgdrTensor* g, const cgdrTensor* cu_seqlens,
                                                     const cgdrTensor* chunk_indices, int64_t chunk_size,
                                                     const cgdrTensor* w, const cgdrTensor* u,
                                                     const cgdrTensor* g_cum, const cgdrWyOptions* options,
                                                     uint64_t* workspace_size, cgdrWyExecutor** executor)
{
    return build_wy(k, v, beta, g, cu_seqlens, chunk_indices, chunk_size, w, u, g_cum, options, workspace_size,
                    executor);
}

void cgdrDestroyWyExecutor(cgdrWyExecutor* executor)
{
    if (executor && executor->magic == kMagicWy) {
        executor->magic = 0;
        delete executor;
    }
}

cgdrStatus cgdrChunkGatedDeltaRuleWY(void* workspace, uint64_t workspace_size, cgdrWyExecutor* executor,
                                     void* stream_ptr)
{
    if (!executor || executor->magic != kMagicWy) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    struct Guard {
        cgdrWyExecutor* e;
        ~Guard() { cgdrDestroyWyExecutor(e); }
    } guard{executor};
    if (!workspace) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace must not be NULL");
    if (workspace_size < kHeader) return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace must hold 256 bytes");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace must be 256-byte aligned");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    cudaError_t e = cudaMemsetAsync(workspace, 0, kHeader, stream);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    return cgdr::host::wy_enqueue(executor, static_cast<int*>(workspace), stream);
}

}  // extern "C"

namespace cgdr {
namespace host {

cgdrStatus wy_enqueue(const cgdrWyExecutor* executor, int* status, cudaStream_t stream)
{
    WyArgs args;
    memset(&args, 0, sizeof(args));
    const WyParams& p = executor->p;
    cgdrStatus st;
    {
        const cgdrTensor& t = executor->tk;
        const int64_t size[4] = {p.K, p.HK, p.T, p.B}, stride[4] = {1, t.strides[2], t.strides[1], t.strides[0]};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&args.maps.k, t.data, 4, size, stride, box, "k"))) return st;
    }
    {
        const cgdrTensor& t = executor->tv;
        const int64_t size[4] = {p.V, p.H, p.T, p.B}, stride[4] = {1, t.strides[2], t.strides[1], t.strides[0]};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&args.maps.v, t.data, 4, size, stride, box, "v"))) return st;
    }
    args.p = p;
    args.p.status = status;
    cudaError_t e = cudaSuccess;
    if (executor->grid == 0) return CGDR_STATUS_SUCCESS;
    if (p.K == 128)
        e = p.V == 128 ? launch_wy<128, 128>(args, executor->grid, stream) : launch_wy<128, 64>(args, executor->grid, stream);
    else
        e = p.V == 128 ? launch_wy<64, 128>(args, executor->grid, stream) : launch_wy<64, 64>(args, executor->grid, stream);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "WY kernel launch: %s", cudaGetErrorString(e));
    return CGDR_STATUS_SUCCESS;
}

}  // namespace host
}  // namespace cgdr
