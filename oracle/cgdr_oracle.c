/*
 * CPU oracle for ChunkGatedDeltaRuleFwdH -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, the smoke()
 * entry of __graft_entry__.py and the cpu_baseline / --impl reference legs of
 * bench.py may load it.  The product path (the CUDA library under the
 * package's csrc/) never links or calls it.
 *
 * It restates, in plain C, the two published semantics of the op:
 *
 *  1. CGDR_ORACLE_REFERENCE -- the normative PyTorch reference of the
 *     contest, with its explicit fp16/bf16 rounding points and a bf16 state
 *     carried between chunks:
 *       ChunkGatedDeltaRuleFwdH_problem_290_template/docs/problem.txt:81-167 (run)
 *       ChunkGatedDeltaRuleFwdH_problem_290_template/code/tests/golden/generate_golden.py:350-440
 *     (run_reference, the validated restatement the golden fixtures come from).
 *     Parity is pinned against fixtures produced by that function
 *     (tests/golden/make_golden.py).
 *
 *  2. CGDR_ORACLE_FP32_STATE -- the vLLM/fla Triton kernel
 *       docs/problem.txt:272-432 (chunk_gated_delta_rule_fwd_kernel_h_blockdim64)
 *     with an fp32 state, bf16 MMA operands when the I/O is bf16, safe_exp
 *     gating and an fp32 final state.  With fp32 I/O the operand casts are
 *     no-ops and the whole recurrence runs in fp32/fp64.  This mode has no
 *     golden vectors in the reference (the Triton text is not runnable on CPU
 *     and the op accepts bf16 only), so for fp32 I/O parity is unpinned.
 *
 * Sums are accumulated in double and rounded once to fp32, which matches
 * torch's CPU bf16 GEMM (fp32 accumulate, one rounding to bf16) except for
 * rare last-bit differences in the fp32 sum.
 *
 * Layout (the fla / north-star layout, all contiguous):
 *   k [B,T,HK,K]   w [B,T,H,K]   u [B,T,H,V]   g [B,T,H] (fp32)
 *   h0/final [N,H,K,V]           h [B,NT,H,K,V]   v_new [B,T,H,V]
 * Varlen (cu_seqlens != NULL) requires B == 1; sequences never share state.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define CGDR_ORACLE_REFERENCE 0
#define CGDR_ORACLE_FP32_STATE 1

#define DT_BF16 1
#define DT_F32 2

/* ---- scalar conversions ------------------------------------------------ */

static inline float bf16_to_f32(uint16_t b)
{
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* float -> bf16, round to nearest even; NaN stays NaN (quietened). */
static inline uint16_t f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* float -> fp16 (RNE, overflow to inf) -> float: torch's plain .to(float16). */
static inline float round_f16(float f) { return (float)(_Float16)f; }

/* cast_to_float16: finite overflow saturates to +-65504, inf/NaN are kept.
 * generate_golden.py:287-292, problem.txt:169-173. */
static inline float cast_f16(float f)
{
    if (isinf(f) || isnan(f)) return round_f16(f);
    float r = round_f16(f);
    if (r > 65504.0f) r = 65504.0f;
    if (r < -65504.0f) r = -65504.0f;
    return r;
}

/* torch.nan_to_num(x, nan=0.0, posinf=inf, neginf=-inf) */
static inline float nan_to_zero(float f) { return isnan(f) ? 0.0f : f; }

static inline float load_io(const void* p, int dt, int64_t i)
{
    return dt == DT_BF16 ? bf16_to_f32(((const uint16_t*)p)[i]) : ((const float*)p)[i];
}

static inline void store_io(void* p, int dt, int64_t i, float v)
{
    if (dt == DT_BF16)
        ((uint16_t*)p)[i] = f32_to_bf16(v);
    else
        ((float*)p)[i] = v;
}

typedef struct {
    int64_t B, T, HK, H, K, V;
    int64_t N;            /* sequences */
    int64_t NT;           /* total chunks (h's chunk dimension) */
    int io_dtype;         /* dtype of k, w, u, v_new, h */
    int h0_dtype;         /* 0 = absent */
    int final_dtype;      /* 0 = not stored */
    int mode;             /* CGDR_ORACLE_* */
    int use_g;            /* fp32-state mode only: g == None disables gating */
    int64_t chunk;        /* 64 */
} oracle_dims_t;

/* One (sequence, value head) recurrence.  All scratch is per call. */
static void run_task(const oracle_dims_t* d, const void* k, const void* w, const void* u,
                     const float* g, const void* h0, void* h, void* v_new, void* fin,
                     int64_t b, int64_t bos, int64_t eos, int64_t boh, int64_t n, int64_t hv)
{
    const int64_t K = d->K, V = d->V, H = d->H, HK = d->HK, BT = d->chunk;
    const int64_t kh = hv / (H / HK);  /* key head: generate_golden.py:410-412 */
    const int64_t T = d->T;
    float* S = (float*)calloc((size_t)(K * V), sizeof(float));
    float* Sb = (float*)malloc((size_t)(K * V) * sizeof(float));   /* MMA1 operand */
    float* vd = (float*)malloc((size_t)(BT * V) * sizeof(float));  /* MMA2 operand */
    double* acc = (double*)malloc((size_t)(K > BT ? K : BT) * (size_t)V * sizeof(double));
    float gate[64];

    /* initial state: generate_golden.py:385-390; problem.txt:338-346 */
    if (h0) {
        for (int64_t i = 0; i < K * V; ++i) {
            float x = load_io(h0, d->h0_dtype, (n * H + hv) * K * V + i);
            S[i] = d->mode == CGDR_ORACLE_REFERENCE ? round_bf16(x) : x;
        }
    }
    const int64_t L = eos - bos;
    const int64_t nchunks = (L + BT - 1) / BT;
    for (int64_t c = 0; c < nchunks; ++c) {
        const int64_t t0 = bos + c * BT;
        const int64_t len = (t0 + BT < eos ? t0 + BT : eos) - t0;
        const int64_t gc = boh + c;
        /* h[:, chunk] = state before the chunk: generate_golden.py:400 */
        for (int64_t i = 0; i < K * V; ++i)
            store_io(h, d->io_dtype, (((b * d->NT + gc) * H + hv) * K * V) + i, S[i]);

        /* token (b, t) -> row offsets in the [B,T,*,*] tensors */
#define ROW_W(t) ((((b) * T + (t)) * H + hv) * K)
#define ROW_K(t) ((((b) * T + (t)) * HK + kh) * K)
#define ROW_U(t) ((((b) * T + (t)) * H + hv) * V)
#define G_AT(t) (g[((b) * T + (t)) * H + hv])

        if (d->mode == CGDR_ORACLE_REFERENCE) {
            /* ws = w_sel @ state, bf16 GEMM -> bf16 -> fp16, NaN -> 0
             * generate_golden.py:414-417 */
            for (int64_t i = 0; i < len; ++i) {
                for (int64_t j = 0; j < V; ++j) acc[j] = 0.0;
                for (int64_t kk = 0; kk < K; ++kk) {
                    const double a = load_io(w, d->io_dtype, ROW_W(t0 + i) + kk);
                    const float* srow = S + kk * V;
                    for (int64_t j = 0; j < V; ++j) acc[j] += a * srow[j];
                }
                const float gl = G_AT(t0 + len - 1);
                /* gate = fp16(exp(g_last - g)): generate_golden.py:423-424 */
                const float gt = cast_f16(expf(gl - G_AT(t0 + i)));
                for (int64_t j = 0; j < V; ++j) {
                    const float ws = nan_to_zero(round_f16(round_bf16((float)acc[j])));
                    /* v_new = fp16(fp16(u) - ws): generate_golden.py:418-421 */
                    const float uu = cast_f16(load_io(u, d->io_dtype, ROW_U(t0 + i) + j));
                    const float vn = cast_f16(uu - ws);
                    /* v_output = bf16(v_new_fp16): generate_golden.py:436 */
                    if (v_new) store_io(v_new, d->io_dtype, ROW_U(t0 + i) + j, vn);
                    /* v_decay = bf16(fp16(v_new * gate)): generate_golden.py:425-426 */
                    vd[i * V + j] = round_bf16(cast_f16(vn * gt));
                }
            }
            /* h_decay = fp16(fp16(state) * exp(fp16(g_last))): generate_golden.py:428-431 */
            const float gl = G_AT(t0 + len - 1);
            const float alpha = round_f16(expf(cast_f16(gl)));
            /* update = k_sel^T @ v_decay, bf16 GEMM -> bf16 -> fp16, NaN -> 0;
             * state = bf16(bf16(h_decay) + bf16(update)): generate_golden.py:433-441 */
            for (int64_t kk = 0; kk < K; ++kk) {
                for (int64_t j = 0; j < V; ++j) acc[j] = 0.0;
                for (int64_t i = 0; i < len; ++i) {
                    const double a = load_io(k, d->io_dtype, ROW_K(t0 + i) + kk);
                    const float* vrow = vd + i * V;
                    for (int64_t j = 0; j < V; ++j) acc[j] += a * vrow[j];
                }
                float* srow = S + kk * V;
                for (int64_t j = 0; j < V; ++j) {
                    const float hd = cast_f16(cast_f16(srow[j]) * alpha);
                    const float up = nan_to_zero(round_f16(round_bf16((float)acc[j])));
                    srow[j] = round_bf16(round_bf16(hd) + round_bf16(up));
                }
            }
        } else {
            /* Triton semantics: problem.txt:353-422 */
            const int bf = d->io_dtype == DT_BF16;
            for (int64_t i = 0; i < K * V; ++i) Sb[i] = bf ? round_bf16(S[i]) : S[i];
            const float gl = d->use_g ? G_AT(t0 + len - 1) : 0.0f;
            for (int64_t i = 0; i < len; ++i) {
                for (int64_t j = 0; j < V; ++j) acc[j] = 0.0;
                for (int64_t kk = 0; kk < K; ++kk) {
                    const double a = load_io(w, d->io_dtype, ROW_W(t0 + i) + kk);
                    const float* srow = Sb + kk * V;
                    for (int64_t j = 0; j < V; ++j) acc[j] += a * srow[j];
                }
                /* b_g = safe_exp(g_last - g): problem.txt:272-274, 377-385 */
                float x = gl - (d->use_g ? G_AT(t0 + i) : 0.0f);
                gate[i] = d->use_g ? expf(x <= 0.0f ? x : -INFINITY) : 1.0f;
                for (int64_t j = 0; j < V; ++j) {
                    const float vn = load_io(u, d->io_dtype, ROW_U(t0 + i) + j) - (float)acc[j];
                    if (v_new) store_io(v_new, d->io_dtype, ROW_U(t0 + i) + j, vn);
                    const float vg = vn * gate[i];
                    vd[i * V + j] = bf ? round_bf16(vg) : vg;
                }
            }
            const float alpha = d->use_g ? expf(gl) : 1.0f;
            for (int64_t kk = 0; kk < K; ++kk) {
                for (int64_t j = 0; j < V; ++j) acc[j] = 0.0;
                for (int64_t i = 0; i < len; ++i) {
                    const double a = load_io(k, d->io_dtype, ROW_K(t0 + i) + kk);
                    const float* vrow = vd + i * V;
                    for (int64_t j = 0; j < V; ++j) acc[j] += a * vrow[j];
                }
                float* srow = S + kk * V;
                for (int64_t j = 0; j < V; ++j) srow[j] = (float)((double)(srow[j] * alpha) + acc[j]);
            }
        }
#undef ROW_W
#undef ROW_K
#undef ROW_U
#undef G_AT
    }
    if (fin) {
        for (int64_t i = 0; i < K * V; ++i)
            store_io(fin, d->final_dtype, (n * H + hv) * K * V + i, S[i]);
    }
    free(S);
    free(Sb);
    free(vd);
    free(acc);
}

/*
 * Entry point.  Returns 0 on success, -1 on a shape error.
 * cu_seqlens: int64 [N+1] or NULL (fixed length: N = B, each batch row is one
 * sequence of length T).  chunk_offsets are recomputed as the cumulative sum
 * of ceil(len/64) (generate_golden.py:275-284).
 * n_threads <= 0 uses every available thread.
 */
int cgdr_oracle_fwd_h(int64_t B, int64_t T, int64_t HK, int64_t H, int64_t K, int64_t V,
                      const void* k, const void* w, const void* u, const float* g,
                      const void* h0, const int64_t* cu_seqlens, int64_t N,
                      void* h, void* v_new, void* fin,
                      int io_dtype, int h0_dtype, int final_dtype, int mode, int use_g,
                      int n_threads)
{
    if (B <= 0 || T < 0 || HK <= 0 || H <= 0 || H % HK != 0 || K <= 0 || V <= 0) return -1;
    if (cu_seqlens && B != 1) return -1;
    if (mode == CGDR_ORACLE_REFERENCE && !g) return -1;
    oracle_dims_t d;
    d.B = B; d.T = T; d.HK = HK; d.H = H; d.K = K; d.V = V;
    d.chunk = 64;
    d.io_dtype = io_dtype; d.h0_dtype = h0 ? h0_dtype : 0;
    d.final_dtype = fin ? final_dtype : 0;
    d.mode = mode;
    d.use_g = g != NULL && use_g;
    int64_t* offs = (int64_t*)malloc((size_t)(cu_seqlens ? N + 1 : B + 1) * sizeof(int64_t));
    if (cu_seqlens) {
        offs[0] = 0;
        for (int64_t n = 0; n < N; ++n) {
            const int64_t L = cu_seqlens[n + 1] - cu_seqlens[n];
            if (L < 0) { free(offs); return -1; }
            offs[n + 1] = offs[n] + (L + 63) / 64;
        }
        d.N = N;
        d.NT = offs[N];
    } else {
        d.N = B;
        d.NT = (T + 63) / 64;
    }
    const int64_t tasks = d.N * H;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t task = 0; task < tasks; ++task) {
        const int64_t n = task / H, hv = task % H;
        int64_t b, bos, eos, boh;
        if (cu_seqlens) {
            b = 0; bos = cu_seqlens[n]; eos = cu_seqlens[n + 1]; boh = offs[n];
        } else {
            b = n; bos = 0; eos = T; boh = 0;
        }
        run_task(&d, k, w, u, g, h0, h, v_new, fin, b, bos, eos, boh, n, hv);
    }
    free(offs);
    return 0;
}

int cgdr_oracle_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
