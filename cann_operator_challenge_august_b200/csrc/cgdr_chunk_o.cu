// Host side of include/cgdr_chunk_o.h: validation, plan, tensor maps and the
// launch of the chunk-output kernel.  No device memory is allocated here.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <new>

#include "../../include/cgdr_chunk_o.h"
#include "host_stages.cuh"
#include "host_util.cuh"
#include "kernel_chunk_o.cuh"

using namespace cgdr;
using namespace cgdr::host;

struct cgdrChunkOExecutor {
    uint32_t magic;
    ChunkOParams p;
    cgdrTensor tq, tk, tv, th, to;
    int64_t grid;
};

namespace {

constexpr uint32_t kMagicO = 0xC6D20C01u;
constexpr uint64_t kHeader = 256;
constexpr int kStagesO = 2;

// SMs of the current device (148 on B200); the plan falls back to that
// figure when no device is visible (phase 1 runs on hosts without a GPU).
int64_t sm_count()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        n > 0)
        return n;
    cudaGetLastError();
    return 148;
}

cgdrStatus build_o(const cgdrTensor* q, const cgdrTensor* k, const cgdrTensor* v, const cgdrTensor* h,
                   const cgdrTensor* g, const cgdrTensor* cu, const cgdrTensor* ci, double scale, int64_t chunk_size,
                   const cgdrTensor* o, const cgdrChunkOOptions* opt, uint64_t* ws_size, cgdrChunkOExecutor** out)
{
    if (!ws_size || !out) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace_size and executor must not be NULL");
    *out = nullptr;
    if (!present(q) || !present(k) || !present(v) || !present(h) || !present(o))
        return fail(CGDR_STATUS_NULL_ARGUMENT, "q, k, v_new, h and o are required");
    const bool has_cu = present(cu), has_ci = present(ci);
    if (has_cu != has_ci)
        return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens and chunk_indices must be both present or both absent");
    cgdrStatus st;
    if ((st = check_rank(q, 4, "q")) || (st = check_rank(k, 4, "k")) || (st = check_rank(v, 4, "v_new")) ||
        (st = check_rank(h, 5, "h")) || (st = check_rank(o, 4, "o")))
        return st;
    if (present(g) && (st = check_rank(g, 3, "g"))) return st;
    if (has_cu && ((st = check_rank(cu, 1, "cu_seqlens")) || (st = check_rank(ci, 2, "chunk_indices")))) return st;
    for (const cgdrTensor* t : {q, k, v, h, o})
        if (t->dtype != CGDR_DT_BF16) return fail(CGDR_STATUS_BAD_DTYPE, "q, k, v_new, h and o must be bfloat16");
    if (present(g) && g->dtype != CGDR_DT_FLOAT32) return fail(CGDR_STATUS_BAD_DTYPE, "g must be float32");
    if (has_cu && (cu->dtype != CGDR_DT_INT64 || ci->dtype != CGDR_DT_INT64))
        return fail(CGDR_STATUS_BAD_DTYPE, "cu_seqlens and chunk_indices must be int64");
    if (chunk_size != kChunk)
        return fail(CGDR_STATUS_BAD_CHUNK_SIZE, "chunk_size must be 64, got %lld", static_cast<long long>(chunk_size));

    const int64_t B = q->shape[0], T = q->shape[1], HK = q->shape[2], K = q->shape[3];
    const int64_t H = v->shape[2], V = v->shape[3];
    if (B <= 0 || T < 0 || HK <= 0 || K <= 0 || H <= 0 || V <= 0)
        return fail(CGDR_STATUS_BAD_SHAPE, "dimensions must be positive");
    if (!shape_is(k, {B, T, HK, K})) return fail(CGDR_STATUS_BAD_SHAPE, "k must have the shape of q [B, T, HK, K]");
    if (v->shape[0] != B || v->shape[1] != T) return fail(CGDR_STATUS_BAD_SHAPE, "v_new must have shape [B, T, HV, V]");
    if (H % HK != 0) return fail(CGDR_STATUS_BAD_SHAPE, "HV must be divisible by HK");
    if (!shape_is(o, {B, T, H, V})) return fail(CGDR_STATUS_BAD_SHAPE, "o must have shape [B, T, HV, V]");
    if (present(g) && !shape_is(g, {B, T, H})) return fail(CGDR_STATUS_BAD_SHAPE, "g must have shape [B, T, HV]");
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
    if (!shape_is(h, {B, NT, H, K, V})) return fail(CGDR_STATUS_BAD_SHAPE, "h must have shape [B, NT, HV, K, V]");
    for (const cgdrTensor* t : {q, k, v, h, o})
        if ((st = check_inner_contiguous(t, "q/k/v_new/h/o"))) return st;
    if (!(K == 64 || K == 128) || V % 64 != 0)
        return fail(CGDR_STATUS_UNSUPPORTED, "chunk output is built for K in {64, 128} and V a multiple of 64");
    for (const cgdrTensor* t : {q, k, v, h, o})
        if (!tma_aligned(t))
            return fail(CGDR_STATUS_BAD_STRIDE, "q, k, v_new, h and o need 16-byte aligned bases and strides");
    if (T >= (int64_t(1) << 31) || NT >= (int64_t(1) << 31))
        return fail(CGDR_STATUS_UNSUPPORTED, "T and NT must fit in 31 bits");

    cgdrChunkOExecutor* ex = new (std::nothrow) cgdrChunkOExecutor();
    if (!ex) return fail(CGDR_STATUS_UNSUPPORTED, "out of host memory");
    ex->magic = kMagicO;
    ChunkOParams& p = ex->p;
    memset(&p, 0, sizeof(p));
    p.g = present(g) ? static_cast<const float*>(g->data) : nullptr;
    p.o = static_cast<__nv_bfloat16*>(o->data);
    p.cu_seqlens = has_cu ? static_cast<const int64_t*>(cu->data) : nullptr;
    p.chunk_indices = has_cu ? static_cast<const int64_t*>(ci->data) : nullptr;
    p.B = B; p.T = T; p.H = H; p.HK = HK; p.K = K; p.V = V; p.N = N; p.NT = NT;
    p.nt_per_seq = (T + kChunk - 1) / kChunk;
    if (present(g)) { p.g_sb = g->strides[0]; p.g_st = g->strides[1]; p.g_sh = g->strides[2]; }
    p.o_sb = o->strides[0]; p.o_st = o->strides[1]; p.o_sh = o->strides[2];
    const int vt = (V % 128 == 0) ? 128 : 64;
    p.n_vtiles = static_cast<int32_t>(V / vt);
    p.varlen = has_cu ? 1 : 0;
    p.scale = static_cast<float>(scale > 0.0 ? scale : 1.0 / std::sqrt(static_cast<double>(K)));
    const int32_t tmo = opt && opt->wait_timeout_ms > 0 ? opt->wait_timeout_ms : 2000;
    p.timeout_ns = static_cast<uint64_t>(tmo) * 1000000ull;
    ex->tq = *q; ex->tk = *k; ex->tv = *v; ex->th = *h; ex->to = *o;
    p.n_tiles = rows * H * p.n_vtiles;
    // persistent: one CTA per SM (or per tile when there are fewer tiles)
    ex->grid = p.n_tiles < sm_count() ? p.n_tiles : sm_count();
    *ws_size = kHeader;
    *out = ex;
    g_err[0] = '\0';
    return CGDR_STATUS_SUCCESS;
}

cgdrStatus build_maps_o(const cgdrChunkOExecutor* ex, ChunkOMaps* m)
{
    const ChunkOParams& p = ex->p;
    cgdrStatus st;
    {
        const cgdrTensor& t = ex->tq;
        const int64_t size[4] = {p.K, p.HK, p.T, p.B}, stride[4] = {1, t.strides[2], t.strides[1], t.strides[0]};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&m->q, t.data, 4, size, stride, box, "q"))) return st;
    }
    {
        const cgdrTensor& t = ex->tk;
        const int64_t size[4] = {p.K, p.HK, p.T, p.B}, stride[4] = {1, t.strides[2], t.strides[1], t.strides[0]};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&m->k, t.data, 4, size, stride, box, "k"))) return st;
    }
    {
        const cgdrTensor& t = ex->tv;
        const int64_t size[4] = {p.V, p.H, p.T, p.B}, stride[4] = {1, t.strides[2], t.strides[1], t.strides[0]};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&m->v, t.data, 4, size, stride, box, "v_new"))) return st;
    }
    {
        const cgdrTensor& t = ex->th;
        const int64_t size[5] = {p.V, p.K, p.H, p.NT, p.B};
        const int64_t stride[5] = {1, t.strides[3], t.strides[2], t.strides[1], t.strides[0]};
        const uint32_t box[5] = {64, static_cast<uint32_t>(p.K), 1, 1, 1};
        if ((st = make_map(&m->h, t.data, 5, size, stride, box, "h"))) return st;
    }
    return CGDR_STATUS_SUCCESS;
}

template <int K_, int VT>
cudaError_t launch_o(const ChunkOArgs& args, int64_t grid, cudaStream_t stream)
{
    using Cfg = ChunkOConfig<K_, VT, kStagesO>;
    auto kern = chunk_o_tc_kernel<K_, VT, kStagesO>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(grid), Cfg::kThreads, Cfg::kSmemBytes, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace

extern "C" {

cgdrStatus cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize(const cgdrTensor* q, const cgdrTensor* k,
                                                       const cgdrTensor* v_new, const cgdrTensor* h,
                                                       const cgdrTensor* g, const cgdrTensor* cu_seqlens,
                                                       const cgdrTensor* chunk_indices, double scale,
                                                       int64_t chunk_size, const cgdrTensor* o,
                                                       const cgdrChunkOOptions* options, uint64_t* workspace_size,
                                                       cgdrChunkOExecutor** executor)
{
    return build_o(q, k, v_new, h, g, cu_seqlens, chunk_indices, scale, chunk_size, o, options, workspace_size,
                   executor);
}

void cgdrDestroyChunkOExecutor(cgdrChunkOExecutor* executor)
{
    if (executor && executor->magic == kMagicO) {
        executor->magic = 0;
        delete executor;
    }
}

int64_t cgdrChunkOGridSize(const cgdrChunkOExecutor* executor)
{
    return (executor && executor->magic == kMagicO) ? executor->grid : -1;
}

cgdrStatus cgdrChunkGatedDeltaRuleFwdO(void* workspace, uint64_t workspace_size, cgdrChunkOExecutor* executor,
                                       void* stream_ptr)
{
    if (!executor || executor->magic != kMagicO) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    struct Guard {
        cgdrChunkOExecutor* e;
        ~Guard() { cgdrDestroyChunkOExecutor(e); }
    } guard{executor};
    if (!workspace) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace must not be NULL");
    if (workspace_size < kHeader) return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace must hold 256 bytes");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace must be 256-byte aligned");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    cudaError_t e = cudaMemsetAsync(workspace, 0, kHeader, stream);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    return cgdr::host::chunk_o_enqueue(executor, static_cast<int*>(workspace), stream);
}

}  // extern "C"

namespace cgdr {
namespace host {

cgdrStatus chunk_o_enqueue(const cgdrChunkOExecutor* executor, int* status, cudaStream_t stream)
{
    ChunkOArgs args;
    memset(&args, 0, sizeof(args));
    cgdrStatus st = build_maps_o(executor, &args.maps);
    if (st) return st;
    args.p = executor->p;
    args.p.status = status;
    cudaError_t e = cudaSuccess;
    if (executor->grid == 0) return CGDR_STATUS_SUCCESS;
    const ChunkOParams& p = executor->p;
    const int vt = static_cast<int>(p.V / p.n_vtiles);
    if (p.K == 128)
        e = vt == 128 ? launch_o<128, 128>(args, executor->grid, stream) : launch_o<128, 64>(args, executor->grid, stream);
    else
        e = vt == 128 ? launch_o<64, 128>(args, executor->grid, stream) : launch_o<64, 64>(args, executor->grid, stream);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "chunk output kernel launch: %s", cudaGetErrorString(e));
    return CGDR_STATUS_SUCCESS;
}

}  // namespace host
}  // namespace cgdr
