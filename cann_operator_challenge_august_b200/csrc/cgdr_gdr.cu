// Host side of include/cgdr_gdr.h: the chunked Gated DeltaNet forward
// operator composed of the WY, recurrence and chunk-output kernels, with the
// reference's argument checks (ref/chunk_gated_delta_rule/op_host/
// chunk_gated_delta_rule_tiling.cpp:375-632 and op_api/
// aclnn_chunk_gated_delta_rule.cpp:64-96).  No device memory is allocated.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <new>

#include "../../include/cgdr_chunk_o.h"
#include "../../include/cgdr_gdr.h"
#include "../../include/cgdr_varlen.h"
#include "../../include/cgdr_wy.h"
#include "common.cuh"
#include "host_stages.cuh"
#include "host_util.cuh"

using namespace cgdr;
using namespace cgdr::host;

namespace cgdr {

// Sequence metadata from actualSeqLengths (one block): cu_seqlens (int64
// [B+1]) and chunk_indices (int64 [nt_max, 2], rows of (sequence, chunk);
// rows past the last chunk are (-1, -1) padding).  Lengths that are negative
// or do not sum to T set status bit 0x2; every write stays inside nt_max rows.
__global__ void __launch_bounds__(256) gdr_meta_kernel(const int32_t* asl, int64_t B, int64_t T, int64_t nt_max,
                                                       int64_t* cu, int64_t* chunk_base, int64_t* ci, int* status)
{
    __shared__ int bad;
    if (threadIdx.x == 0) {
        int64_t run = 0, chunks = 0;
        int b = 0;
        cu[0] = 0;
        chunk_base[0] = 0;
        for (int64_t n = 0; n < B; ++n) {
            int64_t L = asl[n];
            if (L < 0) {
                b = 1;
                L = 0;
            }
            run += L;
            chunks += (L + kChunk - 1) / kChunk;
            cu[n + 1] = run;
            chunk_base[n + 1] = chunks;
        }
        if (run != T || chunks > nt_max) b = 1;
        bad = b;
        if (b && status) atomicOr(status, 0x2);
    }
    __syncthreads();
    for (int64_t n = threadIdx.x; n < B; n += blockDim.x) {
        const int64_t c0 = chunk_base[n], c1 = chunk_base[n + 1];
        for (int64_t r = c0; r < c1 && r < nt_max; ++r) {
            ci[2 * r] = n;
            ci[2 * r + 1] = r - c0;
        }
    }
    const int64_t used = bad ? 0 : chunk_base[B];
    for (int64_t r = used + threadIdx.x; r < nt_max; r += blockDim.x) {
        ci[2 * r] = -1;
        ci[2 * r + 1] = -1;
    }
}

// Chunk list from cu_seqlens (one block of 256 threads): chunk_offsets [N+1]
// and chunk_indices [capacity, 2] with (-1, -1) padding rows.  Thread t owns a
// contiguous range of sequences; a scan of the 256 partial chunk counts gives
// each range its first row.  An invalid cu_seqlens (not non-decreasing from 0,
// or more chunks than capacity) leaves every row padding.
__global__ void __launch_bounds__(256) chunk_list_kernel(const int64_t* cu, int64_t N, int64_t chunk,
                                                         int64_t capacity, int64_t* offsets, int64_t* ci)
{
    __shared__ int64_t part[256];
    __shared__ int bad;
    __shared__ int64_t total;
    const int tid = threadIdx.x;
    if (tid == 0) bad = cu[0] != 0;
    __syncthreads();
    const int64_t per = (N + 255) / 256;
    const int64_t lo = tid * per, hi = lo + per < N ? lo + per : N;
    int64_t sum = 0;
    for (int64_t n = lo; n < hi; ++n) {
        const int64_t L = cu[n + 1] - cu[n];
        if (L < 0) bad = 1;
        sum += L > 0 ? (L + chunk - 1) / chunk : 0;
    }
    part[tid] = sum;
    __syncthreads();
    if (tid == 0) {
        int64_t run = 0;
        for (int i = 0; i < 256; ++i) {
            const int64_t v = part[i];
            part[i] = run;
            run += v;
        }
        if (run > capacity) bad = 1;
        total = bad ? 0 : run;
    }
    __syncthreads();
    int64_t row = part[tid];
    for (int64_t n = lo; n < hi; ++n) {
        const int64_t L = cu[n + 1] - cu[n];
        const int64_t nc = L > 0 ? (L + chunk - 1) / chunk : 0;
        if (offsets) offsets[n] = row;
        if (!bad)
            for (int64_t c = 0; c < nc; ++c) {
                ci[2 * (row + c)] = n;
                ci[2 * (row + c) + 1] = c;
            }
        row += nc;
    }
    // the last thread's running count is the total (its range is the last one)
    if (offsets && tid == 255) offsets[N] = row;
    for (int64_t r = total + tid; r < capacity; r += 256) {
        ci[2 * r] = -1;
        ci[2 * r + 1] = -1;
    }
}

// Zero-padding of the head dimension for Dk, Dv outside {64, 128}: the
// kernels run at the next supported width and the padded columns carry exact
// zeros through every product and sum (k k^T, T' k, w S, k^T v_dec, q S), so
// the result equals the unpadded arithmetic.
//   src [R0, R1, D] (strides s0, s1, 1) -> dst [R0, R1, Dp] contiguous, zeros past D
__global__ void __launch_bounds__(256) pad_heads_kernel(const __nv_bfloat16* src, int64_t s0, int64_t s1, int64_t R0,
                                                        int64_t R1, int64_t D, __nv_bfloat16* dst, int64_t Dp)
{
    const int64_t n = R0 * R1 * Dp;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t d = i % Dp, r = i / Dp, r1 = r % R1, r0 = r / R1;
        dst[i] = d < D ? src[r0 * s0 + r1 * s1 + d] : __float2bfloat16(0.0f);
    }
}

//   dst [R0, R1, D] (strides s0, s1, 1) <- src [R0, R1, Dp] contiguous, first D columns
__global__ void __launch_bounds__(256) unpad_heads_kernel(const __nv_bfloat16* src, int64_t Dp, int64_t R0, int64_t R1,
                                                          int64_t D, __nv_bfloat16* dst, int64_t s0, int64_t s1)
{
    const int64_t n = R0 * R1 * D;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t d = i % D, r = i / D, r1 = r % R1, r0 = r / R1;
        dst[r0 * s0 + r1 * s1 + d] = src[r * Dp + d];
    }
}

// states: [B, Nv, Dv, Dk] (any strides, bf16 or fp32) <-> [B, Nv, Kp, Vp] fp32 contiguous
__global__ void __launch_bounds__(256) pad_state_kernel(const void* src, int32_t dt, int64_t s0, int64_t s1, int64_t sv,
                                                        int64_t sk, int64_t B, int64_t Nv, int64_t Dv, int64_t Dk,
                                                        float* dst, int64_t Kp, int64_t Vp)
{
    const int64_t n = B * Nv * Kp * Vp;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t vv = i % Vp, kk = (i / Vp) % Kp, bn = i / (Vp * Kp), nn = bn % Nv, b = bn / Nv;
        float x = 0.0f;
        if (kk < Dk && vv < Dv) {
            const int64_t at = b * s0 + nn * s1 + vv * sv + kk * sk;
            x = dt == CGDR_DT_FLOAT32 ? static_cast<const float*>(src)[at]
                                      : __bfloat162float(static_cast<const __nv_bfloat16*>(src)[at]);
        }
        dst[i] = x;
    }
}

__global__ void __launch_bounds__(256) unpad_state_kernel(const float* src, int64_t Kp, int64_t Vp, int64_t B,
                                                          int64_t Nv, int64_t Dv, int64_t Dk, void* dst, int32_t dt,
                                                          int64_t s0, int64_t s1, int64_t sv, int64_t sk)
{
    const int64_t n = B * Nv * Dv * Dk;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t kk = i % Dk, vv = (i / Dk) % Dv, bn = i / (Dk * Dv), nn = bn % Nv, b = bn / Nv;
        const float x = src[((b * Nv + nn) * Kp + kk) * Vp + vv];
        const int64_t at = b * s0 + nn * s1 + vv * sv + kk * sk;
        if (dt == CGDR_DT_FLOAT32)
            static_cast<float*>(dst)[at] = x;
        else
            static_cast<__nv_bfloat16*>(dst)[at] = __float2bfloat16_rn(x);
    }
}

}  // namespace cgdr

struct cgdrGdrExecutor {
    uint32_t magic;
    cgdrTensor q, k, v, beta, h0, asl, g, out, fin;
    bool has_g;
    float scale;
    int64_t B, T, Nk, Nv, Dk, Dv, nt_max;
    int64_t Kp, Vp;  // head widths the kernels run at (Dk, Dv padded up to 64 or 128)
    bool fused;      // recurrence and chunk output in one kernel (no h / v_new in the workspace)
    // workspace layout (byte offsets)
    uint64_t off_cu, off_cb, off_ci, off_meta, off_gc, off_w, off_u, off_vn, off_h, total;
    uint64_t off_qp, off_kp, off_vp, off_op, off_h0p, off_finp;  // padding buffers (Kp != Dk or Vp != Dv)
};

namespace {

constexpr uint32_t kMagicGdr = 0xC6D2D0A5u;
constexpr uint64_t kHeader = 256;
constexpr int64_t kMaxHeads = 64;    // tiling.cpp:504-507
constexpr int64_t kMaxHeadDim = 128; // tiling.cpp:509-512

cgdrTensor view(void* data, int32_t dtype, std::initializer_list<int64_t> shape, std::initializer_list<int64_t> strides)
{
    cgdrTensor t;
    memset(&t, 0, sizeof(t));
    t.data = data;
    t.dtype = dtype;
    t.ndim = static_cast<int32_t>(shape.size());
    int i = 0;
    for (int64_t x : shape) t.shape[i++] = x;
    i = 0;
    for (int64_t x : strides) t.strides[i++] = x;
    return t;
}

cgdrTensor contiguous(void* data, int32_t dtype, std::initializer_list<int64_t> shape)
{
    cgdrTensor t = view(data, dtype, shape, shape);
    int64_t s = 1;
    for (int i = t.ndim - 1; i >= 0; --i) {
        t.strides[i] = s;
        s *= t.shape[i];
    }
    return t;
}

bool has_empty(const cgdrTensor* t)
{
    for (int i = 0; i < t->ndim; ++i)
        if (t->shape[i] == 0) return true;
    return false;
}

bool sixteen(const cgdrTensor* t)
{
    if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return false;
    for (int i = 0; i < t->ndim - 1; ++i)
        if ((t->strides[i] * 2) % 16 != 0) return false;
    return t->strides[t->ndim - 1] == 1;
}

cgdrStatus build_gdr(const cgdrTensor* q, const cgdrTensor* k, const cgdrTensor* v, const cgdrTensor* beta,
                     const cgdrTensor* h0, const cgdrTensor* asl, const cgdrTensor* g, float scale,
                     const cgdrTensor* out, const cgdrTensor* fin, const cgdrGdrOptions* options, uint64_t* ws_size,
                     cgdrGdrExecutor** exo)
{
    const int32_t path = options ? options->path : CGDR_GDR_PATH_AUTO;
    if (path != CGDR_GDR_PATH_AUTO && path != CGDR_GDR_PATH_FUSED && path != CGDR_GDR_PATH_THREE_KERNELS)
        return fail(CGDR_STATUS_UNSUPPORTED, "unknown path %d", static_cast<int>(path));
    if (!ws_size || !exo) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspaceSize and executor must not be NULL");
    *exo = nullptr;
    // aclnn_chunk_gated_delta_rule.cpp:64-76: every tensor but g is required
    if (!present(q) || !present(k) || !present(v) || !present(h0) || !present(beta) || !present(asl) ||
        !present(out) || !present(fin))
        return fail(CGDR_STATUS_NULL_ARGUMENT,
                    "query, key, value, initialState, beta, actualSeqLengths, out and finalState are required");
    const bool has_g = present(g);
    // dtypes (aclnn_chunk_gated_delta_rule.cpp:54-95)
    for (const cgdrTensor* t : {q, k, v, beta, out})
        if (t->dtype != CGDR_DT_BF16) return fail(CGDR_STATUS_BAD_DTYPE, "query, key, value, beta and out must be bfloat16");
    for (const cgdrTensor* t : {h0, fin})
        if (t->dtype != CGDR_DT_BF16 && t->dtype != CGDR_DT_FLOAT32)
            return fail(CGDR_STATUS_BAD_DTYPE, "initialState and finalState must be bfloat16 or float32");
    if (asl->dtype != CGDR_DT_INT32) return fail(CGDR_STATUS_BAD_DTYPE, "actualSeqLengths must be int32");
    if (has_g && g->dtype != CGDR_DT_FLOAT32) return fail(CGDR_STATUS_BAD_DTYPE, "g must be float32");
    // ranks (tiling.cpp:535-541)
    cgdrStatus st;
    if ((st = check_rank(q, 3, "query")) || (st = check_rank(k, 3, "key")) || (st = check_rank(v, 3, "value")) ||
        (st = check_rank(beta, 2, "beta")) || (st = check_rank(h0, 4, "initial_state")) ||
        (st = check_rank(asl, 1, "actual_seq_lengths")) || (st = check_rank(out, 3, "out")) ||
        (st = check_rank(fin, 4, "final_state")))
        return st;
    if (has_g && (st = check_rank(g, 2, "g"))) return st;
    // dimensions (tiling.cpp:495-518)
    const int64_t T = q->shape[0], Nk = q->shape[1], Dk = q->shape[2], Nv = v->shape[1], Dv = v->shape[2];
    const int64_t B = h0->shape[0];
    if (T <= 0 || B <= 0 || Nk <= 0 || Dk <= 0 || Nv <= 0 || Dv <= 0)
        return fail(CGDR_STATUS_BAD_SHAPE,
                    "T, B, Nk, Dk, Nv, Dv should be greater than 0, but T=%lld, B=%lld, Nk=%lld, Dk=%lld, Nv=%lld, Dv=%lld",
                    (long long)T, (long long)B, (long long)Nk, (long long)Dk, (long long)Nv, (long long)Dv);
    if (Nk > kMaxHeads || Nv > kMaxHeads)
        return fail(CGDR_STATUS_BAD_SHAPE, "nk and nv should no bigger than 64, but nk is %lld, nv is %lld", (long long)Nk,
                    (long long)Nv);
    if (Dv > kMaxHeadDim || Dk > kMaxHeadDim)
        return fail(CGDR_STATUS_BAD_SHAPE, "dv and dk should be no bigger than 128, but dv is %lld, dk is %lld",
                    (long long)Dv, (long long)Dk);
    if (Nv % Nk != 0)
        return fail(CGDR_STATUS_BAD_SHAPE, "nv should be an integer multiple of nk, but nv is %lld, nk is %lld",
                    (long long)Nv, (long long)Nk);
    // expected shapes (tiling.cpp:375-490)
    if (!shape_is(k, {T, Nk, Dk})) return fail(CGDR_STATUS_BAD_SHAPE, "The shape of key parameter is not expected");
    if (!shape_is(v, {T, Nv, Dv})) return fail(CGDR_STATUS_BAD_SHAPE, "The shape of value parameter is not expected");
    if (!shape_is(beta, {T, Nv})) return fail(CGDR_STATUS_BAD_SHAPE, "The shape of beta parameter is not expected");
    if (!shape_is(h0, {B, Nv, Dv, Dk}))
        return fail(CGDR_STATUS_BAD_SHAPE, "The shape of initial_state parameter is not expected");
    if (!shape_is(asl, {B})) return fail(CGDR_STATUS_BAD_SHAPE, "The shape of actual_seq_lengths parameter is not expected");
    if (!shape_is(out, {T, Nv, Dv})) return fail(CGDR_STATUS_BAD_SHAPE, "The shape of out parameter is not expected");
    if (!shape_is(fin, {B, Nv, Dv, Dk}))
        return fail(CGDR_STATUS_BAD_SHAPE, "The shape of final_state parameter is not expected");
    if (has_g && !shape_is(g, {T, Nv})) return fail(CGDR_STATUS_BAD_SHAPE, "The shape of g parameter is not expected");
    // empty tensors (tiling.cpp:567-590)
    for (const cgdrTensor* t : {q, k, v, beta, h0, asl, out, fin})
        if (has_empty(t)) return fail(CGDR_STATUS_BAD_SHAPE, "empty tensors are not supported");
    // the kernels run at Dk, Dv in {64, 128}; other widths go through zero-padded copies
    const int64_t Kp = Dk <= 64 ? 64 : 128, Vp = Dv <= 64 ? 64 : 128;
    const bool padK = Kp != Dk, padV = Vp != Dv;
    for (const cgdrTensor* t : {q, k})
        if (t->strides[2] != 1 || (!padK && !sixteen(t)))
            return fail(CGDR_STATUS_BAD_STRIDE,
                        "query, key, value and out need a contiguous last dimension and 16-byte aligned strides");
    for (const cgdrTensor* t : {v, out})
        if (t->strides[2] != 1 || (!padV && !sixteen(t)))
            return fail(CGDR_STATUS_BAD_STRIDE,
                        "query, key, value and out need a contiguous last dimension and 16-byte aligned strides");
    if (asl->strides[0] != 1 && B > 1) return fail(CGDR_STATUS_BAD_STRIDE, "actualSeqLengths must be contiguous");
    if (T >= (int64_t(1) << 31)) return fail(CGDR_STATUS_UNSUPPORTED, "T must fit in 31 bits");

    cgdrGdrExecutor* ex = new (std::nothrow) cgdrGdrExecutor();
    if (!ex) return fail(CGDR_STATUS_UNSUPPORTED, "out of host memory");
    ex->magic = kMagicGdr;
    ex->q = *q; ex->k = *k; ex->v = *v; ex->beta = *beta; ex->h0 = *h0; ex->asl = *asl;
    ex->out = *out; ex->fin = *fin;
    ex->has_g = has_g;
    if (has_g) ex->g = *g;
    ex->scale = scale > 0.0f ? scale : static_cast<float>(1.0 / std::sqrt(static_cast<double>(Dk)));
    ex->B = B; ex->T = T; ex->Nk = Nk; ex->Nv = Nv; ex->Dk = Dk; ex->Dv = Dv;
    ex->Kp = Kp; ex->Vp = Vp;
    ex->nt_max = (T + kChunk - 1) / kChunk + B - 1;
    // the fused kernel runs K = 128 (Dk in (64, 128]); AUTO takes it once the
    // (sequence, head) tasks fill half the SMs, below which the separate
    // recurrence (64-column tiles) and the chunk-parallel output spread wider
    const bool fused_applies = Kp == 128;
    if (path == CGDR_GDR_PATH_FUSED && !fused_applies) {
        delete ex;
        return fail(CGDR_STATUS_UNSUPPORTED, "the fused path needs 64 < Dk <= 128, got Dk=%lld", (long long)Dk);
    }
    ex->fused = path == CGDR_GDR_PATH_FUSED || (path == CGDR_GDR_PATH_AUTO && fused_applies && B * Nv >= 74);
    uint64_t off = kHeader;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = off;
        off += align256(bytes);
        return at;
    };
    ex->off_cu = take(8 * static_cast<uint64_t>(B + 1));
    ex->off_cb = take(8 * static_cast<uint64_t>(B + 1));
    ex->off_ci = take(16 * static_cast<uint64_t>(ex->nt_max));
    // the recurrence's varlen metadata: chunk base [N+1] and launch order [N], int32
    ex->off_meta = take(align256(4 * static_cast<uint64_t>(B + 1)) + align256(4 * static_cast<uint64_t>(B)));
    ex->off_gc = take(4 * static_cast<uint64_t>(T * Nv));
    ex->off_w = take(2 * static_cast<uint64_t>(T * Nv * Kp));
    ex->off_u = take(2 * static_cast<uint64_t>(T * Nv * Vp));
    ex->off_vn = ex->off_h = 0;
    if (!ex->fused) {
        ex->off_vn = take(2 * static_cast<uint64_t>(T * Nv * Vp));
        ex->off_h = take(2 * static_cast<uint64_t>(ex->nt_max * Nv * Kp * Vp));
    }
    ex->off_qp = ex->off_kp = ex->off_vp = ex->off_op = ex->off_h0p = ex->off_finp = 0;
    if (padK) {
        ex->off_qp = take(2 * static_cast<uint64_t>(T * Nk * Kp));
        ex->off_kp = take(2 * static_cast<uint64_t>(T * Nk * Kp));
    }
    if (padV) {
        ex->off_vp = take(2 * static_cast<uint64_t>(T * Nv * Vp));
        ex->off_op = take(2 * static_cast<uint64_t>(T * Nv * Vp));
    }
    if (padK || padV) {
        ex->off_h0p = take(4 * static_cast<uint64_t>(B * Nv * Kp * Vp));
        ex->off_finp = take(4 * static_cast<uint64_t>(B * Nv * Kp * Vp));
    }
    ex->total = off;
    *ws_size = off;
    *exo = ex;
    g_err[0] = '\0';
    return CGDR_STATUS_SUCCESS;
}

}  // namespace

extern "C" {

cgdrStatus cgdrChunkGatedDeltaRuleGetWorkspaceSize(const cgdrTensor* query, const cgdrTensor* key,
                                                   const cgdrTensor* value, const cgdrTensor* beta,
                                                   const cgdrTensor* initialState, const cgdrTensor* actualSeqLengths,
                                                   const cgdrTensor* gOptional, float scaleValue,
                                                   const cgdrTensor* out, const cgdrTensor* finalState,
                                                   uint64_t* workspaceSize, cgdrGdrExecutor** executor)
{
    return build_gdr(query, key, value, beta, initialState, actualSeqLengths, gOptional, scaleValue, out, finalState,
                     nullptr, workspaceSize, executor);
}

cgdrStatus cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx(const cgdrTensor* query, const cgdrTensor* key,
                                                     const cgdrTensor* value, const cgdrTensor* beta,
                                                     const cgdrTensor* initialState,
                                                     const cgdrTensor* actualSeqLengths, const cgdrTensor* gOptional,
                                                     float scaleValue, const cgdrTensor* out,
                                                     const cgdrTensor* finalState, const cgdrGdrOptions* options,
                                                     uint64_t* workspaceSize, cgdrGdrExecutor** executor)
{
    return build_gdr(query, key, value, beta, initialState, actualSeqLengths, gOptional, scaleValue, out, finalState,
                     options, workspaceSize, executor);
}

cgdrStatus cgdrGetGdrPath(const cgdrGdrExecutor* executor, int32_t* path)
{
    if (!executor || executor->magic != kMagicGdr) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    if (!path) return fail(CGDR_STATUS_NULL_ARGUMENT, "path must not be NULL");
    *path = executor->fused ? CGDR_GDR_PATH_FUSED : CGDR_GDR_PATH_THREE_KERNELS;
    return CGDR_STATUS_SUCCESS;
}

void cgdrDestroyGdrExecutor(cgdrGdrExecutor* executor)
{
    if (executor && executor->magic == kMagicGdr) {
        executor->magic = 0;
        delete executor;
    }
}

cgdrStatus cgdrChunkGatedDeltaRule(void* workspace, uint64_t workspaceSize, cgdrGdrExecutor* executor, void* stream_ptr)
{
    if (!executor || executor->magic != kMagicGdr) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    struct Guard {
        cgdrGdrExecutor* e;
        ~Guard() { cgdrDestroyGdrExecutor(e); }
    } guard{executor};
    const cgdrGdrExecutor& ex = *executor;
    if (!workspace) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace must not be NULL");
    if (workspaceSize < ex.total)
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace of %llu bytes is smaller than the %llu required",
                    (unsigned long long)workspaceSize, (unsigned long long)ex.total);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace must be 256-byte aligned");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int* status = reinterpret_cast<int*>(ws);
    const int64_t T = ex.T, Nk = ex.Nk, Nv = ex.Nv, B = ex.B, NT = ex.nt_max;
    const int64_t Dk = ex.Kp, Dv = ex.Vp;  // the widths the kernels run at
    const bool padK = ex.Kp != ex.Dk, padV = ex.Vp != ex.Dv, padS = padK || padV;

    // views: the TND tensors as [1, T, heads, dim] (a packed varlen batch), the
    // [B, Nv, Dv, Dk] states as [B, Nv, K=Dk, V=Dv] by their strides; padded
    // copies in the workspace where a width is not 64 or 128
    const cgdrTensor q4 = padK ? contiguous(ws + ex.off_qp, CGDR_DT_BF16, {1, T, Nk, Dk})
                               : view(ex.q.data, CGDR_DT_BF16, {1, T, Nk, Dk},
                                      {T * ex.q.strides[0], ex.q.strides[0], ex.q.strides[1], ex.q.strides[2]});
    const cgdrTensor k4 = padK ? contiguous(ws + ex.off_kp, CGDR_DT_BF16, {1, T, Nk, Dk})
                               : view(ex.k.data, CGDR_DT_BF16, {1, T, Nk, Dk},
                                      {T * ex.k.strides[0], ex.k.strides[0], ex.k.strides[1], ex.k.strides[2]});
    const cgdrTensor v4 = padV ? contiguous(ws + ex.off_vp, CGDR_DT_BF16, {1, T, Nv, Dv})
                               : view(ex.v.data, CGDR_DT_BF16, {1, T, Nv, Dv},
                                      {T * ex.v.strides[0], ex.v.strides[0], ex.v.strides[1], ex.v.strides[2]});
    const cgdrTensor o4 = padV ? contiguous(ws + ex.off_op, CGDR_DT_BF16, {1, T, Nv, Dv})
                               : view(ex.out.data, CGDR_DT_BF16, {1, T, Nv, Dv},
                                      {T * ex.out.strides[0], ex.out.strides[0], ex.out.strides[1], ex.out.strides[2]});
    const cgdrTensor b3 = view(ex.beta.data, CGDR_DT_BF16, {1, T, Nv},
                               {T * ex.beta.strides[0], ex.beta.strides[0], ex.beta.strides[1]});
    cgdrTensor g3;
    memset(&g3, 0, sizeof(g3));
    if (ex.has_g) g3 = view(ex.g.data, CGDR_DT_FLOAT32, {1, T, Nv}, {T * ex.g.strides[0], ex.g.strides[0], ex.g.strides[1]});
    const cgdrTensor h0 = padS ? contiguous(ws + ex.off_h0p, CGDR_DT_FLOAT32, {B, Nv, Dk, Dv})
                               : view(ex.h0.data, ex.h0.dtype, {B, Nv, Dk, Dv},
                                      {ex.h0.strides[0], ex.h0.strides[1], ex.h0.strides[3], ex.h0.strides[2]});
    const cgdrTensor fin = padS ? contiguous(ws + ex.off_finp, CGDR_DT_FLOAT32, {B, Nv, Dk, Dv})
                                : view(ex.fin.data, ex.fin.dtype, {B, Nv, Dk, Dv},
                                       {ex.fin.strides[0], ex.fin.strides[1], ex.fin.strides[3], ex.fin.strides[2]});
    // workspace tensors
    const cgdrTensor cu = contiguous(ws + ex.off_cu, CGDR_DT_INT64, {B + 1});
    const cgdrTensor ci = contiguous(ws + ex.off_ci, CGDR_DT_INT64, {NT, 2});
    const cgdrTensor gc = contiguous(ws + ex.off_gc, CGDR_DT_FLOAT32, {1, T, Nv});
    const cgdrTensor w = contiguous(ws + ex.off_w, CGDR_DT_BF16, {1, T, Nv, Dk});
    const cgdrTensor u = contiguous(ws + ex.off_u, CGDR_DT_BF16, {1, T, Nv, Dv});
    // on the fused path h and v_new have no buffer: the recurrence plan gets a
    // placeholder h view (shape checks only; nothing reads or writes it) and no v_new
    const cgdrTensor vn = contiguous(ws + ex.off_vn, CGDR_DT_BF16, {1, T, Nv, Dv});
    const cgdrTensor h = contiguous(ws + ex.off_h, CGDR_DT_BF16, {1, NT, Nv, Dk, Dv});

    // plans of the three stages (host only)
    cgdrWyExecutor* e_wy = nullptr;
    cgdrExecutor* e_h = nullptr;
    cgdrChunkOExecutor* e_o = nullptr;
    struct Owned {
        cgdrWyExecutor*& a;
        cgdrExecutor*& b;
        cgdrChunkOExecutor*& c;
        ~Owned()
        {
            cgdrDestroyWyExecutor(a);
            cgdrDestroyExecutor(b);
            cgdrDestroyChunkOExecutor(c);
        }
    } owned{e_wy, e_h, e_o};
    uint64_t sz = 0;
    cgdrStatus st;
    if ((st = cgdrChunkGatedDeltaRuleWYGetWorkspaceSize(&k4, &v4, &b3, ex.has_g ? &g3 : nullptr, &cu, &ci, kChunk, &w, &u,
                                                        &gc, nullptr, &sz, &e_wy)))
        return st;
    cgdrFwdHOptions opt;
    memset(&opt, 0, sizeof(opt));
    opt.layout = CGDR_LAYOUT_TOKEN_MAJOR;
    opt.numerics = CGDR_NUMERICS_FP32_STATE;
    if ((st = cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx(&k4, &w, &u, &gc, &h0, &cu, &ci, nullptr, kChunk, &h,
                                                            ex.fused ? nullptr : &vn, &fin, &opt, &sz, &e_h)))
        return st;
    if (ex.fused && !fwd_ho_applies(e_h)) return fail(CGDR_STATUS_UNSUPPORTED, "internal: fused plan not applicable");
    if (fwd_h_meta_bytes(e_h) > align256(4 * static_cast<uint64_t>(B + 1)) + align256(4 * static_cast<uint64_t>(B)))
        return fail(CGDR_STATUS_UNSUPPORTED, "internal: recurrence metadata does not fit");
    if (!ex.fused && (st = cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize(&q4, &k4, &vn, &h, &gc, &cu, &ci, ex.scale,
                                                                       kChunk, &o4, nullptr, &sz, &e_o)))
        return st;

    // enqueue: status word, metadata, WY, recurrence, chunk output (one stream)
    cudaError_t e = cudaMemsetAsync(ws, 0, kHeader, stream);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    gdr_meta_kernel<<<1, 256, 0, stream>>>(static_cast<const int32_t*>(ex.asl.data), B, T, NT,
                                           reinterpret_cast<int64_t*>(ws + ex.off_cu),
                                           reinterpret_cast<int64_t*>(ws + ex.off_cb),
                                           reinterpret_cast<int64_t*>(ws + ex.off_ci), status);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return fail(CGDR_STATUS_CUDA_ERROR, "metadata kernel launch: %s", cudaGetErrorString(e));
    auto blocks = [](int64_t n) { return static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 8)); };
    if (padK) {
        pad_heads_kernel<<<blocks(T * Nk * Dk), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(ex.q.data), ex.q.strides[0], ex.q.strides[1], T, Nk, ex.Dk,
            reinterpret_cast<__nv_bfloat16*>(ws + ex.off_qp), Dk);
        pad_heads_kernel<<<blocks(T * Nk * Dk), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(ex.k.data), ex.k.strides[0], ex.k.strides[1], T, Nk, ex.Dk,
            reinterpret_cast<__nv_bfloat16*>(ws + ex.off_kp), Dk);
    }
    if (padV)
        pad_heads_kernel<<<blocks(T * Nv * Dv), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(ex.v.data), ex.v.strides[0], ex.v.strides[1], T, Nv, ex.Dv,
            reinterpret_cast<__nv_bfloat16*>(ws + ex.off_vp), Dv);
    if (padS)
        pad_state_kernel<<<blocks(B * Nv * Dk * Dv), 256, 0, stream>>>(
            ex.h0.data, ex.h0.dtype, ex.h0.strides[0], ex.h0.strides[1], ex.h0.strides[2], ex.h0.strides[3], B, Nv,
            ex.Dv, ex.Dk, reinterpret_cast<float*>(ws + ex.off_h0p), Dk, Dv);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return fail(CGDR_STATUS_CUDA_ERROR, "padding kernel launch: %s", cudaGetErrorString(e));
    if ((st = wy_enqueue(e_wy, status, stream))) return st;
    if (ex.fused) {
        if ((st = fwd_ho_enqueue(e_h, &q4, &o4, ex.scale, status, ws + ex.off_meta, stream))) return st;
    } else {
        if ((st = fwd_h_enqueue(e_h, status, ws + ex.off_meta, stream))) return st;
        if ((st = chunk_o_enqueue(e_o, status, stream))) return st;
    }
    if (padV)
        unpad_heads_kernel<<<blocks(T * Nv * ex.Dv), 256, 0, stream>>>(
            reinterpret_cast<const __nv_bfloat16*>(ws + ex.off_op), Dv, T, Nv, ex.Dv,
            static_cast<__nv_bfloat16*>(ex.out.data), ex.out.strides[0], ex.out.strides[1]);
    if (padS)
        unpad_state_kernel<<<blocks(B * Nv * ex.Dv * ex.Dk), 256, 0, stream>>>(
            reinterpret_cast<const float*>(ws + ex.off_finp), Dk, Dv, B, Nv, ex.Dv, ex.Dk, ex.fin.data, ex.fin.dtype,
            ex.fin.strides[0], ex.fin.strides[1], ex.fin.strides[2], ex.fin.strides[3]);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return fail(CGDR_STATUS_CUDA_ERROR, "unpadding kernel launch: %s", cudaGetErrorString(e));
    return CGDR_STATUS_SUCCESS;
}

}  // extern "C"

extern "C" cgdrStatus cgdrPrepareChunkIndices(const cgdrTensor* cu_seqlens, int64_t chunk_size,
                                              const cgdrTensor* chunk_indices, const cgdrTensor* chunk_offsets,
                                              void* stream)
{
    if (!present(cu_seqlens) || !present(chunk_indices))
        return fail(CGDR_STATUS_NULL_ARGUMENT, "cu_seqlens and chunk_indices are required");
    cgdrStatus st;
    if ((st = check_rank(cu_seqlens, 1, "cu_seqlens")) || (st = check_rank(chunk_indices, 2, "chunk_indices"))) return st;
    if (present(chunk_offsets) && (st = check_rank(chunk_offsets, 1, "chunk_offsets"))) return st;
    if (cu_seqlens->dtype != CGDR_DT_INT64 || chunk_indices->dtype != CGDR_DT_INT64 ||
        (present(chunk_offsets) && chunk_offsets->dtype != CGDR_DT_INT64))
        return fail(CGDR_STATUS_BAD_DTYPE, "cu_seqlens, chunk_indices and chunk_offsets must be int64");
    if (chunk_size <= 0) return fail(CGDR_STATUS_BAD_CHUNK_SIZE, "chunk_size must be positive");
    const int64_t N = cu_seqlens->shape[0] - 1;
    if (N < 1) return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens needs at least two entries");
    if (chunk_indices->shape[1] != 2) return fail(CGDR_STATUS_BAD_SHAPE, "chunk_indices must have shape [capacity, 2]");
    if (present(chunk_offsets) && chunk_offsets->shape[0] != N + 1)
        return fail(CGDR_STATUS_BAD_SHAPE, "chunk_offsets must have N + 1 entries");
    if ((cu_seqlens->shape[0] > 1 && cu_seqlens->strides[0] != 1) || chunk_indices->strides[1] != 1 ||
        chunk_indices->strides[0] != 2 || (present(chunk_offsets) && chunk_offsets->strides[0] != 1))
        return fail(CGDR_STATUS_BAD_STRIDE, "the metadata tensors must be contiguous");
    const int64_t capacity = chunk_indices->shape[0];
    if (capacity == 0) return CGDR_STATUS_SUCCESS;
    chunk_list_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const int64_t*>(cu_seqlens->data), N, chunk_size, capacity,
        present(chunk_offsets) ? static_cast<int64_t*>(chunk_offsets->data) : nullptr,
        static_cast<int64_t*>(chunk_indices->data));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "chunk list kernel launch: %s", cudaGetErrorString(e));
    return CGDR_STATUS_SUCCESS;
}
