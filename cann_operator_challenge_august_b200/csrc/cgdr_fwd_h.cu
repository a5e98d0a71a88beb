// Host side of the C ABI declared in include/cgdr_fwd_h.h: argument
// validation (the counterpart of the reference's shape inference,
// code/op_host/chunk_gated_delta_rule_fwd_h_infershape.cpp:135-299), the
// launch plan (the counterpart of its tiling function,
// code/op_host/chunk_gated_delta_rule_fwd_h_tiling.cpp:152-261), tensor-map
// encoding and the launches.  No device memory is allocated here.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "../../include/cgdr_fwd_h.h"
#include "common.cuh"
#include "host_stages.cuh"
#include "host_util.cuh"
#include "kernel_simt.cuh"
#include "kernel_ho.cuh"
#include "kernel_tc.cuh"

using namespace cgdr;
using namespace cgdr::host;

namespace {

constexpr int64_t kMaxTokens = 256 * 1024;  // infershape.cpp:32
constexpr int64_t kMaxValueHeads = 128;     // infershape.cpp:33
constexpr int64_t kMaxKeyHeads = 32;        // infershape.cpp:34
constexpr int64_t kMinHeadDim = 32;         // infershape.cpp:35
constexpr int64_t kMaxHeadDim = 256;        // infershape.cpp:36
constexpr int64_t kMaxSequences = 4;        // infershape.cpp:31
constexpr uint64_t kHeaderBytes = 256;      // workspace: device status word

}  // namespace

struct cgdrExecutor {
    uint32_t magic;
    FwdHParams p;
    cgdrFwdHPlan plan;
    int32_t force_kernel;
    int32_t has_v;
    // tensor-map source descriptions (byte strides) for the TMA path
    cgdrTensor tk, tw, tu, tv, th;
};

namespace {

constexpr uint32_t kMagic = 0xC6D2F0A1u;

struct Dims {
    int64_t B, T, HK, HV, K, V, N, NT;
};

int io_of(int32_t dt) { return dt == CGDR_DT_BF16 ? kBF16 : (dt == CGDR_DT_FLOAT32 ? kF32 : 0); }

// Whether a tensor-core plan runs the sixteen-warp epilogue (K tile 128, 128-column tiles,
// reference arithmetic): its v_new staging is per warp, 32 columns with the 64-byte swizzle.
bool tc_quarters(const cgdrFwdHPlan& pl)
{
    return pl.kernel == 1 && pl.v_tile == 128 && pl.block == TcConfig<128, 128, 3, 4>::kThreads;
}

// K tile of the tensor-core kernel for head width K (0: no tensor-core kernel).
int tc_k_tile(int64_t K)
{
    if (K < 8 || K > 256 || K % 8 != 0) return 0;
    return K <= 64 ? 64 : K <= 128 ? 128 : 256;
}

cgdrStatus build(const cgdrTensor* k, const cgdrTensor* w, const cgdrTensor* u, const cgdrTensor* g,
                 const cgdrTensor* h0, const cgdrTensor* cu, const cgdrTensor* ci, const cgdrTensor* co,
                 int64_t chunk_size, const cgdrTensor* h, const cgdrTensor* v, const cgdrTensor* fin,
                 const cgdrFwdHOptions& opt, bool ex, uint64_t* ws_size, cgdrExecutor** out)
{
    if (!ws_size || !out) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace_size and executor must not be NULL");
    *out = nullptr;
    if (!present(k) || !present(w) || !present(u) || !present(h))
        return fail(CGDR_STATUS_NULL_ARGUMENT, "k, w, u and h are required");
    const bool ref = opt.numerics == CGDR_NUMERICS_REFERENCE;
    if (opt.numerics != CGDR_NUMERICS_REFERENCE && opt.numerics != CGDR_NUMERICS_FP32_STATE)
        return fail(CGDR_STATUS_UNSUPPORTED, "unknown numerics mode %d", opt.numerics);
    if (opt.layout != CGDR_LAYOUT_HEAD_MAJOR && opt.layout != CGDR_LAYOUT_TOKEN_MAJOR)
        return fail(CGDR_STATUS_UNSUPPORTED, "unknown layout %d", opt.layout);
    const bool head_major = opt.layout == CGDR_LAYOUT_HEAD_MAJOR;
    if (!present(g) && (ref || !ex)) return fail(CGDR_STATUS_NULL_ARGUMENT, "g is required");
    if (!present(v) && !ex) return fail(CGDR_STATUS_NULL_ARGUMENT, "v is required");
    const bool has_cu = present(cu), has_ci = present(ci);
    if (has_cu != has_ci && (!ex || opt.strict_reference_limits || (has_ci && !has_cu)))
        return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens and chunk_indices must be both present or both absent");

    // ---- ranks (infershape.cpp:149-164)
    cgdrStatus st;
    if ((st = check_rank(k, 4, "k")) || (st = check_rank(w, 4, "w")) || (st = check_rank(u, 4, "u"))) return st;
    if (present(g) && (st = check_rank(g, 3, "g"))) return st;
    if (present(h0) && (st = check_rank(h0, 4, "initial_state"))) return st;
    if (has_cu && (st = check_rank(cu, 1, "cu_seqlens"))) return st;
    if (has_ci && (st = check_rank(ci, 2, "chunk_indices"))) return st;
    if (present(co) && (st = check_rank(co, 1, "chunk_offsets"))) return st;
    if ((st = check_rank(h, 5, "h"))) return st;
    if (present(v) && (st = check_rank(v, 4, "v"))) return st;
    if (present(fin) && (st = check_rank(fin, 4, "final_state"))) return st;

    // ---- dtypes (infershape.cpp:166-181)
    const int io = io_of(k->dtype);
    if (!io || (ref && io != kBF16))
        return fail(CGDR_STATUS_BAD_DTYPE, ref ? "k must be bfloat16" : "k must be bfloat16 or float32");
    if (io_of(w->dtype) != io || io_of(u->dtype) != io || io_of(h->dtype) != io ||
        (present(v) && io_of(v->dtype) != io))
        return fail(CGDR_STATUS_BAD_DTYPE, "w, u, h and v must have the dtype of k");
    if (present(g) && g->dtype != CGDR_DT_FLOAT32) return fail(CGDR_STATUS_BAD_DTYPE, "g must be float32");
    if (present(h0) && !io_of(h0->dtype))
        return fail(CGDR_STATUS_BAD_DTYPE, "initial_state must be bfloat16 or float32");
    if (present(fin) && !io_of(fin->dtype))
        return fail(CGDR_STATUS_BAD_DTYPE, "final_state must be bfloat16 or float32");
    if (!ex) {
        if ((present(h0) && h0->dtype != CGDR_DT_BF16) || (present(fin) && fin->dtype != CGDR_DT_BF16))
            return fail(CGDR_STATUS_BAD_DTYPE, "initial_state and final_state must be bfloat16");
    }
    if ((has_cu && cu->dtype != CGDR_DT_INT64) || (has_ci && ci->dtype != CGDR_DT_INT64) ||
        (present(co) && co->dtype != CGDR_DT_INT64))
        return fail(CGDR_STATUS_BAD_DTYPE, "cu_seqlens, chunk_indices and chunk_offsets must be int64");

    // ---- chunk size (infershape.cpp:183-190)
    if (chunk_size != kChunk) return fail(CGDR_STATUS_BAD_CHUNK_SIZE, "chunk_size must be 64, got %lld",
                                          static_cast<long long>(chunk_size));

    // ---- dimensions
    Dims d;
    d.B = k->shape[0];
    d.T = k->shape[1];
    d.HK = k->shape[2];
    d.K = k->shape[3];
    d.HV = head_major ? u->shape[1] : u->shape[2];
    d.V = u->shape[3];
    const int64_t uT = head_major ? u->shape[2] : u->shape[1];
    if (d.B <= 0 || d.T < 0 || d.HK <= 0 || d.HV <= 0 || d.K <= 0 || d.V <= 0)
        return fail(CGDR_STATUS_BAD_SHAPE, "dimensions must be positive");
    if (u->shape[0] != d.B || uT != d.T) return fail(CGDR_STATUS_BAD_SHAPE, "u must have shape [B, HV, T, V] / [B, T, HV, V]");
    if (!(head_major ? shape_is(w, {d.B, d.HV, d.T, d.K}) : shape_is(w, {d.B, d.T, d.HV, d.K})))
        return fail(CGDR_STATUS_BAD_SHAPE, "w must have shape %s", head_major ? "[B, HV, T, K]" : "[B, T, HV, K]");
    if (present(g) && !(head_major ? shape_is(g, {d.B, d.HV, d.T}) : shape_is(g, {d.B, d.T, d.HV})))
        return fail(CGDR_STATUS_BAD_SHAPE, "g must have shape %s", head_major ? "[B, HV, T]" : "[B, T, HV]");
    if (d.HV % d.HK != 0)
        return fail(CGDR_STATUS_BAD_SHAPE, "HV must be divisible by HK: HV=%lld, HK=%lld",
                    static_cast<long long>(d.HV), static_cast<long long>(d.HK));
    if (d.K > kMaxHeadDim) return fail(CGDR_STATUS_UNSUPPORTED, "K must be <= 256");
    if (opt.strict_reference_limits) {
        if (d.B != 1) return fail(CGDR_STATUS_BAD_SHAPE, "B must be 1, but got %lld", static_cast<long long>(d.B));
        if (d.T <= 0 || d.T > kMaxTokens) return fail(CGDR_STATUS_BAD_SHAPE, "T must be in [1, 262144]");
        if (d.HK > kMaxKeyHeads || d.HV > kMaxValueHeads)
            return fail(CGDR_STATUS_BAD_SHAPE, "HK/HV are out of range: HK=%lld, HV=%lld",
                        static_cast<long long>(d.HK), static_cast<long long>(d.HV));
        if (d.K < kMinHeadDim || d.K > kMaxHeadDim || d.V != d.K)
            return fail(CGDR_STATUS_BAD_SHAPE, "K and V must be equal and in [32, 256], but got K=%lld, V=%lld",
                        static_cast<long long>(d.K), static_cast<long long>(d.V));
    }

    // ---- sequences and chunk count (infershape.cpp:240-288)
    const int64_t nt_min = (d.T + kChunk - 1) / kChunk;
    const int64_t h_nt = head_major ? h->shape[2] : h->shape[1];
    if (has_cu) {
        if (d.B != 1) return fail(CGDR_STATUS_BAD_VARLEN, "variable-length input needs B == 1");
        const int64_t len = cu->shape[0];
        if (len < 2) return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens needs at least two entries");
        if (opt.strict_reference_limits && len > kMaxSequences + 1)
            return fail(CGDR_STATUS_BAD_VARLEN, "cu_seqlens length must be in [2, 5], but got %lld",
                        static_cast<long long>(len));
        d.N = len - 1;
        if (opt.strict_reference_limits && d.N > d.T)
            return fail(CGDR_STATUS_BAD_VARLEN, "The number of non-empty sequences cannot exceed T");
        if (has_ci) {
            if (ci->shape[1] != 2) return fail(CGDR_STATUS_BAD_VARLEN, "chunk_indices must have shape [NT, 2]");
            d.NT = ci->shape[0];
        } else {
            d.NT = h_nt;
        }
        const int64_t nt_max = nt_min + d.N - 1;
        if (d.NT < nt_min || d.NT > nt_max)
            return fail(CGDR_STATUS_BAD_VARLEN, "NT=%lld is impossible for T=%lld and N=%lld; expected range [%lld, %lld]",
                        static_cast<long long>(d.NT), static_cast<long long>(d.T), static_cast<long long>(d.N),
                        static_cast<long long>(nt_min), static_cast<long long>(nt_max));
        if (present(co) && co->shape[0] != d.N + 1)
            return fail(CGDR_STATUS_BAD_VARLEN, "chunk_offsets must have N + 1 entries");
    } else {
        d.N = d.B;
        d.NT = nt_min;
    }
    if (present(h0) && !shape_is(h0, {d.N, d.HV, d.K, d.V}))
        return fail(CGDR_STATUS_BAD_SHAPE, "initial_state must have shape [N, HV, K, V]");
    if (!(head_major ? shape_is(h, {d.B, d.HV, d.NT, d.K, d.V}) : shape_is(h, {d.B, d.NT, d.HV, d.K, d.V})))
        return fail(CGDR_STATUS_BAD_SHAPE, "h must have shape %s", head_major ? "[B, HV, NT, K, V]" : "[B, NT, HV, K, V]");
    if (present(v) && !(head_major ? shape_is(v, {d.B, d.HV, d.T, d.V}) : shape_is(v, {d.B, d.T, d.HV, d.V})))
        return fail(CGDR_STATUS_BAD_SHAPE, "v must have shape %s", head_major ? "[B, HV, T, V]" : "[B, T, HV, V]");
    if (present(fin) && !shape_is(fin, {d.N, d.HV, d.K, d.V}))
        return fail(CGDR_STATUS_BAD_SHAPE, "final_state must have shape [N, HV, K, V]");

    // ---- strides: innermost contiguous
    if ((st = check_inner_contiguous(k, "k")) || (st = check_inner_contiguous(w, "w")) ||
        (st = check_inner_contiguous(u, "u")) || (st = check_inner_contiguous(h, "h")))
        return st;
    if (present(v) && (st = check_inner_contiguous(v, "v"))) return st;
    // initial and final state may be [.., K, V] with any strides (a transposed
    // [.., V, K] view included); they are read and written once per task
    for (const cgdrTensor* t : {h0, fin})
        if (present(t))
            for (int i = 0; i < t->ndim; ++i)
                if (t->strides[i] < 0) return fail(CGDR_STATUS_BAD_STRIDE, "negative stride in a state tensor");
    if (has_cu && cu->shape[0] > 1 && cu->strides[0] != 1) return fail(CGDR_STATUS_BAD_STRIDE, "cu_seqlens must be contiguous");
    if (present(co) && co->shape[0] > 1 && co->strides[0] != 1)
        return fail(CGDR_STATUS_BAD_STRIDE, "chunk_offsets must be contiguous");

    // ---- parameter block
    cgdrExecutor* ex_ = new (std::nothrow) cgdrExecutor();
    if (!ex_) return fail(CGDR_STATUS_UNSUPPORTED, "out of host memory");
    ex_->magic = kMagic;
    FwdHParams& p = ex_->p;
    memset(&p, 0, sizeof(p));
    p.k = k->data;
    p.w = w->data;
    p.u = u->data;
    p.g = present(g) ? static_cast<const float*>(g->data) : nullptr;
    p.h0 = present(h0) ? h0->data : nullptr;
    p.cu_seqlens = has_cu ? static_cast<const int64_t*>(cu->data) : nullptr;
    p.chunk_offsets = present(co) ? static_cast<const int64_t*>(co->data) : nullptr;
    p.h = h->data;
    p.v_new = present(v) ? v->data : nullptr;
    p.final_state = present(fin) ? fin->data : nullptr;
    p.B = d.B; p.T = d.T; p.HK = d.HK; p.H = d.HV; p.K = d.K; p.V = d.V; p.N = d.N; p.NT = d.NT;
    p.k_sb = k->strides[0]; p.k_st = k->strides[1]; p.k_sh = k->strides[2];
    if (head_major) {
        p.w_sb = w->strides[0]; p.w_sh = w->strides[1]; p.w_st = w->strides[2];
        p.u_sb = u->strides[0]; p.u_sh = u->strides[1]; p.u_st = u->strides[2];
        if (present(g)) { p.g_sb = g->strides[0]; p.g_sh = g->strides[1]; p.g_st = g->strides[2]; }
        if (present(v)) { p.v_sb = v->strides[0]; p.v_sh = v->strides[1]; p.v_st = v->strides[2]; }
        p.h_sb = h->strides[0]; p.h_sh = h->strides[1]; p.h_sc = h->strides[2]; p.h_sk = h->strides[3];
    } else {
        p.w_sb = w->strides[0]; p.w_st = w->strides[1]; p.w_sh = w->strides[2];
        p.u_sb = u->strides[0]; p.u_st = u->strides[1]; p.u_sh = u->strides[2];
        if (present(g)) { p.g_sb = g->strides[0]; p.g_st = g->strides[1]; p.g_sh = g->strides[2]; }
        if (present(v)) { p.v_sb = v->strides[0]; p.v_st = v->strides[1]; p.v_sh = v->strides[2]; }
        p.h_sb = h->strides[0]; p.h_sc = h->strides[1]; p.h_sh = h->strides[2]; p.h_sk = h->strides[3];
    }
    if (present(h0)) {
        p.h0_sn = h0->strides[0]; p.h0_sh = h0->strides[1]; p.h0_sk = h0->strides[2]; p.h0_sv = h0->strides[3];
    }
    if (present(fin)) {
        p.f_sn = fin->strides[0]; p.f_sh = fin->strides[1]; p.f_sk = fin->strides[2]; p.f_sv = fin->strides[3];
    }
    p.io_dtype = io;
    p.h0_dtype = present(h0) ? io_of(h0->dtype) : 0;
    p.f_dtype = present(fin) ? io_of(fin->dtype) : 0;
    p.numerics = ref ? 0 : 1;
    p.use_g = present(g) ? 1 : 0;
    p.varlen = has_cu ? 1 : 0;
    p.fault_inject = opt.fault_inject;
    p.timeout_ns = static_cast<uint64_t>(opt.wait_timeout_ms > 0 ? opt.wait_timeout_ms : 2000) * 1000000ull;
    ex_->tk = *k; ex_->tw = *w; ex_->tu = *u; ex_->th = *h;
    if (present(v)) ex_->tv = *v;
    ex_->has_v = present(v);
    ex_->force_kernel = opt.force_kernel;

    // ---- plan (tiling.cpp:215-259)
    cgdrFwdHPlan& pl = ex_->plan;
    memset(&pl, 0, sizeof(pl));
    pl.batch = d.B; pl.total_tokens = d.T; pl.key_heads = d.HK; pl.value_heads = d.HV;
    pl.key_dim = d.K; pl.value_dim = d.V; pl.sequence_count = d.N; pl.chunk_count = d.NT;
    pl.head_ratio = d.HV / d.HK;
    pl.has_initial_state = present(h0); pl.is_varlen = has_cu; pl.store_final_state = present(fin);
    pl.save_new_value = present(v);
    pl.plan_key = pl.has_initial_state | (pl.is_varlen << 1) | (pl.store_final_state << 2);
    pl.numerics = opt.numerics;
    pl.layout = opt.layout;

    // Tensor-core path eligibility: bf16 I/O, K and V multiples of 8 with K <= 256,
    // TMA-describable strides (16-byte multiples) and aligned bases.  The kernel's K
    // tile is the next of 64, 128 and 256: k_c and w_c columns past K arrive
    // zero-filled from the tensor maps, so the padded rows of the state stay zero and
    // are never stored; a V tile that runs past V is clipped the same way.
    auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    auto st16 = [](const cgdrTensor* t) {
        for (int i = 0; i < t->ndim - 1; ++i)
            if ((t->strides[i] * 2) % 16 != 0) return false;
        return true;
    };
    const int kt = tc_k_tile(d.K);
    bool tc_ok = io == kBF16 && kt > 0 && d.V % 8 == 0 && al16(k->data) && al16(w->data) &&
                 al16(u->data) && al16(h->data) && st16(k) && st16(w) && st16(u) && st16(h) &&
                 (!present(v) || (al16(v->data) && st16(v))) && d.T < (int64_t(1) << 31) &&
                 d.NT < (int64_t(1) << 31);
    if (opt.force_kernel == 2) tc_ok = false;
    if (opt.force_kernel == 1 && !tc_ok) {
        delete ex_;
        return fail(CGDR_STATUS_UNSUPPORTED, "tensor-core path requested but not applicable to these shapes/strides");
    }
    if (tc_ok) {
        auto tasks = [&](int vt) { return d.N * d.HV * ((d.V + vt - 1) / vt); };
        int vt = opt.v_tile;
        if (vt == 0) {
            // The narrowest tiles that still fit one CTA per SM: a (sequence, head) chain
            // split over more SMs carries less epilogue work per chunk.  32-column tiles
            // (K tile 128) while they fit, then 64-column ones; beyond one CTA per SM
            // 128-column tiles: on B=4, T=8192, H=32, K=V=128 (256 64-column tasks)
            // they take 0.288 ms against 0.307 ms for two 64-column CTAs per SM.  The
            // K tile 256 runs 64-column tiles only (its shared memory holds no wider).
            if (kt == 256)
                vt = 64;
            else if (kt == 128 && (d.V % 64 != 0 || tasks(32) <= 148))
                vt = 32;
            else
                vt = (d.V % 128 == 0 && tasks(64) > 148) ? 128 : 64;
        }
        if (vt != 32 && vt != 64 && vt != 128) {
            delete ex_;
            return fail(CGDR_STATUS_UNSUPPORTED, "v_tile must be 32, 64 or 128 on the tensor-core path");
        }
        if (vt == 32 && kt != 128) {
            delete ex_;
            return fail(CGDR_STATUS_UNSUPPORTED, "v_tile 32 needs 64 < K <= 128");
        }
        // Two chains per CTA (each column half of the V tile a chain of its own) are
        // built for the K tile 128 with 32- and 128-column tiles.  The automatic plan
        // takes them for the reference arithmetic, whose heavier epilogues then run
        // while the other chain's MMAs do: B=1 T=65536 H=32 1.485 against 1.597 ms,
        // B=4 T=8192 H=32 0.459 against 0.467 ms (sixteen-warp single chain).  The
        // fp32-state chain is bound by the MMA hand-offs, and two chains there only
        // contend for the tensor pipe (1.134 against 1.089 ms; 0.283 against 0.273 ms).
        const bool two_chain_tile = kt == 128 && (vt == 32 || vt == 128);
        const int chains = opt.chains != 0 ? opt.chains : (ref && two_chain_tile ? 2 : 1);
        if (chains != 1 && chains != 2) {
            delete ex_;
            return fail(CGDR_STATUS_UNSUPPORTED, "chains must be 0 (auto), 1 or 2");
        }
        if (chains == 2 && !two_chain_tile) {
            delete ex_;
            return fail(CGDR_STATUS_UNSUPPORTED, "two chains per CTA need 64 < K <= 128 and v_tile 32 or 128");
        }
        pl.chains = chains;
        if (kt == 256 && vt != 64) {
            delete ex_;
            return fail(CGDR_STATUS_UNSUPPORTED, "K > 128 runs 64-column V tiles only");
        }
        pl.kernel = 1;
        pl.v_tile = vt;
        pl.stages = (vt == 64) ? 2 : 3;
        // The reference arithmetic's 128-column tiles (K tile 128) run sixteen epilogue
        // warps (four 32-column quarters per lane quadrant): its epilogues issue about twice
        // the instructions of the fp32-state ones.
        pl.block = kt == 256                      ? TcConfig<256, 64, 2, 2>::kThreads
                   : chains == 2                  ? TcConfig<128, 32, 3, 2, 2>::kThreads  // 11 warps (either width)
                   : (vt == 128 && kt == 128 && ref) ? TcConfig<128, 128, 3, 4>::kThreads
                   : vt == 128                    ? TcConfig<128, 128, 3, 2>::kThreads
                                                  : TcConfig<128, 64, 2, 1>::kThreads;
    } else {
        if (d.K < 1 || d.K > kMaxHeadDim) {
            delete ex_;
            return fail(CGDR_STATUS_UNSUPPORTED, "K=%lld not supported", static_cast<long long>(d.K));
        }
        pl.kernel = 2;
        pl.v_tile = kSimtVT;
        pl.stages = 1;
        pl.block = kSimtThreads;
        pl.smem_bytes = static_cast<int32_t>(simt_smem_bytes(static_cast<int>(d.K)));
    }
    if (pl.chains == 0) pl.chains = 1;
    pl.v_tile_count = (d.V + pl.v_tile - 1) / pl.v_tile;
    // a CTA runs one V tile: one chain, or two of half its width
    pl.task_count = d.N * d.HV * pl.v_tile_count * pl.chains;
    pl.grid = static_cast<int32_t>(d.N * d.HV * pl.v_tile_count);
    p.v_tile = static_cast<int32_t>(pl.v_tile);
    p.n_vtiles = static_cast<int32_t>(pl.v_tile_count);
    if (pl.kernel == 1) {
#define CGDR_SMEM(K_, VT_, ST_, EW_) TcConfig<K_, VT_, ST_, EW_>::kSmemBytes
#define CGDR_SMEM2(K_, VT_) TcConfig<K_, VT_, 3, 2, 2>::kSmemBytes
        if (kt == 256)
            pl.smem_bytes = CGDR_SMEM(256, 64, 2, 2);
        else if (kt == 128)
            pl.smem_bytes = pl.chains == 2    ? (pl.v_tile == 128 ? CGDR_SMEM2(128, 128) : CGDR_SMEM2(128, 32))
                            : pl.v_tile == 128 ? (ref ? CGDR_SMEM(128, 128, 3, 4) : CGDR_SMEM(128, 128, 3, 2))
                            : pl.v_tile == 64  ? CGDR_SMEM(128, 64, 2, 1)
                                               : CGDR_SMEM(128, 32, 3, 1);
        else
            pl.smem_bytes = pl.v_tile == 128 ? CGDR_SMEM(64, 128, 3, 2) : CGDR_SMEM(64, 64, 2, 1);
#undef CGDR_SMEM
#undef CGDR_SMEM2
    }
    uint64_t ws = kHeaderBytes;
    if (has_cu) ws += align256(4 * static_cast<uint64_t>(d.N + 1)) + align256(4 * static_cast<uint64_t>(d.N));
    pl.workspace_bytes = ws;
    *ws_size = ws;
    *out = ex_;
    g_err[0] = '\0';
    return CGDR_STATUS_SUCCESS;
}

// ---- tensor maps ----------------------------------------------------------------

cgdrStatus build_maps(const cgdrExecutor* ex, TcMaps* m)
{
    const FwdHParams& p = ex->p;
    const bool hm = ex->plan.layout == CGDR_LAYOUT_HEAD_MAJOR;
    (void)hm;
    cgdrStatus st;
    {
        const int64_t size[4] = {p.K, p.HK, p.T, p.B}, stride[4] = {1, p.k_sh, p.k_st, p.k_sb};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&m->k, const_cast<void*>(p.k), 4, size, stride, box, "k"))) return st;
    }
    {
        const int64_t size[4] = {p.K, p.H, p.T, p.B}, stride[4] = {1, p.w_sh, p.w_st, p.w_sb};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&m->w, const_cast<void*>(p.w), 4, size, stride, box, "w"))) return st;
    }
    // 32-column tiles move u, v_new and h in 32-column boxes with the 64-byte swizzle,
    // the two 16-column chains in 16-column boxes with the 32-byte swizzle
    const bool sw32 = ex->plan.v_tile == 32 && ex->plan.chains == 2;
    const bool sw64 = ex->plan.v_tile == 32 && !sw32;
    const uint32_t cols = sw32 ? 16 : sw64 ? 32 : 64;
    const int swz = sw32 ? 32 : sw64 ? 64 : 128;
    {
        const int64_t size[4] = {p.V, p.H, p.T, p.B}, stride[4] = {1, p.u_sh, p.u_st, p.u_sb};
        const uint32_t box[4] = {cols, 1, 64, 1};
        if ((st = make_map(&m->u, const_cast<void*>(p.u), 4, size, stride, box, "u", swz))) return st;
    }
    if (p.v_new) {
        // the K tile 256 kernel stages v_new per warp in 32-column regions (64-byte swizzle)
        const bool v32 = sw64 || tc_k_tile(p.K) == 256 || tc_quarters(ex->plan);
        const int64_t size[4] = {p.V, p.H, p.T, p.B}, stride[4] = {1, p.v_sh, p.v_st, p.v_sb};
        const uint32_t box[4] = {sw32 ? 16u : v32 ? 32u : 64u, 1, 16, 1};
        if ((st = make_map(&m->v, p.v_new, 4, size, stride, box, "v", sw32 ? 32 : v32 ? 64 : 128))) return st;
    } else {
        memset(&m->v, 0, sizeof(m->v));
    }
    {
        const int64_t size[5] = {p.V, p.K, p.H, p.NT, p.B}, stride[5] = {1, p.h_sk, p.h_sh, p.h_sc, p.h_sb};
        const uint32_t box[5] = {cols, static_cast<uint32_t>(tc_k_tile(p.K) == 64 ? 16 : 32), 1, 1, 1};
        if ((st = make_map(&m->h, p.h, 5, size, stride, box, "h", swz))) return st;
    }
    return CGDR_STATUS_SUCCESS;
}

template <int K_, int VT, int STAGES, int EW, bool REF, int CH = 1>
cudaError_t launch_tc(const TcArgs& args, int grid, cudaStream_t stream)
{
    using Cfg = TcConfig<K_, VT, STAGES, EW, CH>;
    auto kern = fwd_h_tc_kernel<K_, VT, STAGES, EW, REF, CH>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(args);
    return cudaGetLastError();
}

template <int K_, int VT, int STAGES, int EW, int CH = 1>
cudaError_t launch_tc_numerics(const TcArgs& args, int grid, cudaStream_t stream)
{
    return args.p.numerics == 0 ? launch_tc<K_, VT, STAGES, EW, true, CH>(args, grid, stream)
                                : launch_tc<K_, VT, STAGES, EW, false, CH>(args, grid, stream);
}

}  // namespace

extern "C" {

cgdrStatus cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize(const cgdrTensor* k, const cgdrTensor* w, const cgdrTensor* u,
                                                       const cgdrTensor* g, const cgdrTensor* initial_state,
                                                       const cgdrTensor* cu_seqlens, const cgdrTensor* chunk_indices,
                                                       int64_t chunk_size, const cgdrTensor* h, const cgdrTensor* v,
                                                       const cgdrTensor* final_state, uint64_t* workspace_size,
                                                       cgdrExecutor** executor)
{
    cgdrFwdHOptions opt;
    memset(&opt, 0, sizeof(opt));
    opt.layout = CGDR_LAYOUT_HEAD_MAJOR;
    opt.numerics = CGDR_NUMERICS_REFERENCE;
    return build(k, w, u, g, initial_state, cu_seqlens, chunk_indices, nullptr, chunk_size, h, v, final_state, opt,
                 false, workspace_size, executor);
}

cgdrStatus cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx(const cgdrTensor* k, const cgdrTensor* w, const cgdrTensor* u,
                                                         const cgdrTensor* g, const cgdrTensor* initial_state,
                                                         const cgdrTensor* cu_seqlens,
                                                         const cgdrTensor* chunk_indices,
                                                         const cgdrTensor* chunk_offsets, int64_t chunk_size,
                                                         const cgdrTensor* h, const cgdrTensor* v,
                                                         const cgdrTensor* final_state,
                                                         const cgdrFwdHOptions* options, uint64_t* workspace_size,
                                                         cgdrExecutor** executor)
{
    cgdrFwdHOptions opt;
    memset(&opt, 0, sizeof(opt));
    if (options) opt = *options;
    return build(k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_offsets, chunk_size, h, v, final_state,
                 opt, true, workspace_size, executor);
}

void cgdrDestroyExecutor(cgdrExecutor* executor)
{
    if (executor && executor->magic == kMagic) {
        executor->magic = 0;
        delete executor;
    }
}

cgdrStatus cgdrGetPlan(const cgdrExecutor* executor, cgdrFwdHPlan* plan)
{
    if (!executor || executor->magic != kMagic) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    if (!plan) return fail(CGDR_STATUS_NULL_ARGUMENT, "plan must not be NULL");
    *plan = executor->plan;
    return CGDR_STATUS_SUCCESS;
}

cgdrStatus cgdrChunkGatedDeltaRuleFwdH(void* workspace, uint64_t workspace_size, cgdrExecutor* executor,
                                       void* stream_ptr)
{
    if (!executor || executor->magic != kMagic) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    struct Guard {
        cgdrExecutor* e;
        ~Guard() { cgdrDestroyExecutor(e); }
    } guard{executor};
    const cgdrFwdHPlan& pl = executor->plan;
    if (!workspace) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace must not be NULL");
    if (workspace_size < pl.workspace_bytes)
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace of %llu bytes is smaller than the %llu required",
                    static_cast<unsigned long long>(workspace_size),
                    static_cast<unsigned long long>(pl.workspace_bytes));
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace must be 256-byte aligned");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws, 0, kHeaderBytes, stream);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    return cgdr::host::fwd_h_enqueue(executor, reinterpret_cast<int*>(ws), ws + kHeaderBytes, stream);
}

}  // extern "C"

namespace cgdr {
namespace host {

uint64_t fwd_h_meta_bytes(const cgdrExecutor* ex)
{
    return ex->plan.workspace_bytes - kHeaderBytes;
}

cgdrStatus fwd_h_enqueue(const cgdrExecutor* executor, int* status, uint8_t* meta, cudaStream_t stream)
{
    const cgdrFwdHPlan& pl = executor->plan;
    FwdHParams p = executor->p;
    p.status = status;
    cudaError_t e = cudaSuccess;
    if (p.varlen) {
        int32_t* base = reinterpret_cast<int32_t*>(meta);
        int32_t* order = reinterpret_cast<int32_t*>(meta + align256(4 * static_cast<uint64_t>(p.N + 1)));
        p.seq_chunk_base = base;
        p.seq_order = order;
        varlen_prep_kernel<<<1, 1024, 0, stream>>>(p.cu_seqlens, p.N, p.T, p.NT, base, order, p.status);
        if ((e = cudaGetLastError()) != cudaSuccess)
            return fail(CGDR_STATUS_CUDA_ERROR, "varlen metadata kernel: %s", cudaGetErrorString(e));
    }
    if (pl.task_count == 0) return CGDR_STATUS_SUCCESS;
    if (pl.kernel == 1) {
        TcArgs args;
        memset(&args, 0, sizeof(args));
        cgdrStatus st = build_maps(executor, &args.maps);
        if (st) return st;
        args.p = p;
        const int grid = pl.grid;
        const int kt = tc_k_tile(p.K);
        if (kt == 256)
            e = launch_tc_numerics<256, 64, 2, 2>(args, grid, stream);
        else if (kt == 128 && pl.chains == 2)
            e = pl.v_tile == 128 ? launch_tc_numerics<128, 128, 3, 2, 2>(args, grid, stream)
                                 : launch_tc_numerics<128, 32, 3, 2, 2>(args, grid, stream);
        else if (kt == 128 && tc_quarters(pl))
            e = launch_tc<128, 128, 3, 4, true>(args, grid, stream);
        else if (kt == 128)
            e = pl.v_tile == 128  ? launch_tc_numerics<128, 128, 3, 2>(args, grid, stream)
                : pl.v_tile == 64 ? launch_tc_numerics<128, 64, 2, 1>(args, grid, stream)
                                  : launch_tc_numerics<128, 32, 3, 1>(args, grid, stream);
        else
            e = pl.v_tile == 128 ? launch_tc_numerics<64, 128, 3, 2>(args, grid, stream)
                                 : launch_tc_numerics<64, 64, 2, 1>(args, grid, stream);
        if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "tensor-core kernel launch: %s", cudaGetErrorString(e));
    } else {
        e = cudaFuncSetAttribute(fwd_h_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem_bytes);
        if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        fwd_h_simt_kernel<<<pl.grid, kSimtThreads, pl.smem_bytes, stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess)
            return fail(CGDR_STATUS_CUDA_ERROR, "general kernel launch: %s", cudaGetErrorString(e));
    }
    return CGDR_STATUS_SUCCESS;
}

bool fwd_ho_applies(const cgdrExecutor* ex)
{
    const FwdHParams& p = ex->p;
    return p.K == 128 && (p.V == 64 || p.V == 128) && p.numerics == 1 && p.io_dtype == kBF16 &&
           ex->plan.layout == CGDR_LAYOUT_TOKEN_MAJOR;
}

cgdrStatus fwd_ho_enqueue(const cgdrExecutor* executor, const cgdrTensor* q, const cgdrTensor* o, float scale,
                          int* status, uint8_t* meta, cudaStream_t stream)
{
    if (!fwd_ho_applies(executor))
        return fail(CGDR_STATUS_UNSUPPORTED, "internal: the fused recurrence + output kernel does not cover this plan");
    FwdHParams p = executor->p;
    p.status = status;
    p.h = nullptr;
    p.v_new = nullptr;
    // q [B, T, HK, K] and o [B, T, H, V], token-major like k and u
    if (q->ndim != 4 || o->ndim != 4 || q->strides[3] != 1 || o->strides[3] != 1 || q->shape[3] != p.K ||
        o->shape[3] != p.V || q->shape[2] != p.HK || o->shape[2] != p.H || q->shape[1] != p.T || o->shape[1] != p.T ||
        q->shape[0] != p.B || o->shape[0] != p.B || q->dtype != CGDR_DT_BF16 || o->dtype != CGDR_DT_BF16)
        return fail(CGDR_STATUS_UNSUPPORTED, "internal: q / o views do not match the recurrence plan");
    if ((reinterpret_cast<uintptr_t>(o->data) & 15) || (o->strides[1] % 8) || (o->strides[2] % 8) || (o->strides[0] % 8))
        return fail(CGDR_STATUS_BAD_STRIDE, "out needs 16-byte aligned rows for the fused kernel");
    cudaError_t e = cudaSuccess;
    if (p.varlen) {
        int32_t* base = reinterpret_cast<int32_t*>(meta);
        int32_t* order = reinterpret_cast<int32_t*>(meta + align256(4 * static_cast<uint64_t>(p.N + 1)));
        p.seq_chunk_base = base;
        p.seq_order = order;
        varlen_prep_kernel<<<1, 1024, 0, stream>>>(p.cu_seqlens, p.N, p.T, p.NT, base, order, p.status);
        if ((e = cudaGetLastError()) != cudaSuccess)
            return fail(CGDR_STATUS_CUDA_ERROR, "varlen metadata kernel: %s", cudaGetErrorString(e));
    }
    const int64_t grid = p.N * p.H;
    if (grid == 0) return CGDR_STATUS_SUCCESS;
    HoArgs args;
    memset(&args, 0, sizeof(args));
    cgdrStatus st;
    {
        const int64_t size[4] = {p.K, p.HK, p.T, p.B}, stride[4] = {1, p.k_sh, p.k_st, p.k_sb};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&args.maps.k, const_cast<void*>(p.k), 4, size, stride, box, "k"))) return st;
    }
    {
        const int64_t size[4] = {p.K, p.H, p.T, p.B}, stride[4] = {1, p.w_sh, p.w_st, p.w_sb};
        const uint32_t box[4] = {64, 1, 16, 1};
        if ((st = make_map(&args.maps.w, const_cast<void*>(p.w), 4, size, stride, box, "w"))) return st;
    }
    {
        const int64_t size[4] = {p.K, p.HK, p.T, p.B}, stride[4] = {1, q->strides[2], q->strides[1], q->strides[0]};
        const uint32_t box[4] = {64, 1, 16, 1};
        if ((st = make_map(&args.maps.q, q->data, 4, size, stride, box, "q"))) return st;
    }
    {
        const int64_t size[4] = {p.V, p.H, p.T, p.B}, stride[4] = {1, p.u_sh, p.u_st, p.u_sb};
        const uint32_t box[4] = {64, 1, 64, 1};
        if ((st = make_map(&args.maps.u, const_cast<void*>(p.u), 4, size, stride, box, "u"))) return st;
    }
    {
        const int64_t size[4] = {p.V, p.H, p.T, p.B}, stride[4] = {1, o->strides[2], o->strides[1], o->strides[0]};
        const uint32_t box[4] = {64, 1, 16, 1};
        if ((st = make_map(&args.maps.o, o->data, 4, size, stride, box, "o"))) return st;
    }
    args.p = p;
    args.x.o = static_cast<__nv_bfloat16*>(o->data);
    args.x.o_sb = o->strides[0];
    args.x.o_st = o->strides[1];
    args.x.o_sh = o->strides[2];
    args.x.scale = scale;
    if (p.V == 128) {
        using Cfg = HoConfig<128>;
        e = cudaFuncSetAttribute(fwd_ho_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
        if (e == cudaSuccess) {
            fwd_ho_tc_kernel<128><<<static_cast<unsigned>(grid), Cfg::kThreads, Cfg::kSmemBytes, stream>>>(args);
            e = cudaGetLastError();
        }
    } else {
        using Cfg = HoConfig<64>;
        e = cudaFuncSetAttribute(fwd_ho_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
        if (e == cudaSuccess) {
            fwd_ho_tc_kernel<64><<<static_cast<unsigned>(grid), Cfg::kThreads, Cfg::kSmemBytes, stream>>>(args);
            e = cudaGetLastError();
        }
    }
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "fused recurrence + output kernel launch: %s", cudaGetErrorString(e));
    return CGDR_STATUS_SUCCESS;
}

}  // namespace host
}  // namespace cgdr

extern "C" {

cgdrStatus cgdrReadDeviceStatus(const void* workspace, uint64_t workspace_size, void* stream, int32_t* device_status)
{
    if (!workspace || !device_status) return fail(CGDR_STATUS_NULL_ARGUMENT, "workspace and device_status are required");
    if (workspace_size < kHeaderBytes) return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL, "workspace too small");
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = cudaMemcpy(device_status, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(CGDR_STATUS_CUDA_ERROR, "reading the device status: %s", cudaGetErrorString(e));
    if (*device_status != 0)
        return fail(CGDR_STATUS_DEVICE_ERROR, "device status 0x%x (%s%s)", *device_status,
                    (*device_status & CGDR_DEVICE_WAIT_TIMEOUT) ? "bounded wait expired " : "",
                    (*device_status & CGDR_DEVICE_BAD_VARLEN) ? "inconsistent cu_seqlens" : "");
    return CGDR_STATUS_SUCCESS;
}

const char* cgdrGetLastErrorMessage(void) { return g_err; }

int32_t cgdrGetAbiVersion(void) { return CGDR_ABI_VERSION; }

}  // extern "C"

// ---- phase 2 without allocation ------------------------------------------------------
// The workspace of cgdrChunkGatedDeltaRuleFwdHNoAlloc: one file-scope device
// array per GPU that loads the library.  Host code must not pass the symbol
// itself to a kernel (on the host it is only a stand-in); its device address
// comes from cudaGetSymbolAddress, looked up once per device.

#include <mutex>

namespace {

__device__ __align__(256) uint8_t g_noalloc_scratch[CGDR_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {};

}  // namespace

extern "C" cgdrStatus cgdrChunkGatedDeltaRuleFwdHNoAlloc(cgdrExecutor* executor, void* stream,
                                                        int32_t* device_status)
{
    if (!executor || executor->magic != kMagic) return fail(CGDR_STATUS_BAD_EXECUTOR, "invalid executor");
    if (executor->plan.workspace_bytes > CGDR_NOALLOC_SCRATCH_BYTES) {
        const unsigned long long need = executor->plan.workspace_bytes;
        cgdrDestroyExecutor(executor);
        return fail(CGDR_STATUS_WORKSPACE_TOO_SMALL,
                    "this call needs %llu bytes of scratch; the built-in buffer holds %d "
                    "(use cgdrChunkGatedDeltaRuleFwdH with a caller workspace)",
                    need, CGDR_NOALLOC_SCRATCH_BYTES);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cgdrDestroyExecutor(executor);
        return fail(CGDR_STATUS_CUDA_ERROR, "cudaGetDevice: %s", cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= kMaxDevices) {
        cgdrDestroyExecutor(executor);
        return fail(CGDR_STATUS_UNSUPPORTED, "device ordinal %d exceeds the %d devices this entry point serves", dev,
                    kMaxDevices);
    }
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if (!g_noalloc_addr[dev]) {
            void* addr = nullptr;
            e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
            if (e != cudaSuccess || addr == nullptr) {
                cgdrDestroyExecutor(executor);
                return fail(CGDR_STATUS_CUDA_ERROR, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
            }
            g_noalloc_addr[dev] = addr;
        }
        scratch = g_noalloc_addr[dev];
    }
    // The ordinary phase 2 on the built-in buffer (it clears the status word).
    const cgdrStatus st = cgdrChunkGatedDeltaRuleFwdH(scratch, CGDR_NOALLOC_SCRATCH_BYTES, executor, stream);
    if (st != CGDR_STATUS_SUCCESS || device_status == nullptr) return st;
    return cgdrReadDeviceStatus(scratch, CGDR_NOALLOC_SCRATCH_BYTES, stream, device_status);
}
