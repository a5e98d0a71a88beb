// General-shape kernel: any 16 <= K <= 256, any V, bf16 or fp32 I/O, both
// numerics modes.  One CTA owns one (sequence, value head, 32-column V tile)
// and walks that sequence's chunks in order (the same task split as the
// reference's ProcessTask, op_kernel/chunk_gated_delta_rule_fwd_h.h:421-510).
// The two per-chunk contractions run as CUDA-core FMAs from shared memory.
// It serves shapes and dtypes the tensor-core kernel does not cover (fp32
// I/O, K or V not a multiple of 8, strides TMA cannot describe).
#pragma once

#include "common.cuh"

namespace cgdr {

constexpr int kSimtVT = 32;
constexpr int kSimtThreads = 256;

__host__ __device__ inline size_t simt_smem_bytes(int K)
{
    // S, Sb: [K][VT]; Wc, Kc: [64][K+1]; Vd: [64][VT]; gate: [64]
    return sizeof(float) * (2 * (size_t)K * kSimtVT + 2 * 64 * (size_t)(K + 1) + 64 * kSimtVT + 64);
}

// Decode blockIdx.x into (sequence, value head, V tile).  V tiles of one head
// are adjacent so that they meet the same k/w lines in L2; varlen sequences go
// longest first when the workspace holds an order.
__device__ __forceinline__ void decode_task(const FwdHParams& p, int64_t bid, int64_t& n, int64_t& hv, int64_t& vt)
{
    vt = bid % p.n_vtiles;
    const int64_t rest = bid / p.n_vtiles;
    hv = rest % p.H;
    const int64_t rank = rest / p.H;
    n = (p.varlen && p.seq_order) ? p.seq_order[rank] : rank;
}

__global__ void __launch_bounds__(kSimtThreads) fwd_h_simt_kernel(const __grid_constant__ FwdHParams p)
{
    extern __shared__ float smem[];
    if (p.status && (*reinterpret_cast<volatile int*>(p.status) & 0x2)) return;  // bad varlen metadata
    const int K = static_cast<int>(p.K);
    constexpr int VT = kSimtVT;
    float* S = smem;
    float* Sb = S + K * VT;
    float* Wc = Sb + K * VT;
    float* Kc = Wc + 64 * (K + 1);
    float* Vd = Kc + 64 * (K + 1);
    float* gate = Vd + 64 * VT;
    __shared__ float s_alpha;

    const int tid = threadIdx.x;
    int64_t n, hv, vt;
    decode_task(p, blockIdx.x, n, hv, vt);
    const SeqInfo si = seq_info(p, n);
    const int64_t kh = hv / (p.H / p.HK);
    const int64_t v0 = vt * VT;
    const int vcount = static_cast<int>(p.V - v0 < VT ? p.V - v0 : VT);
    const bool ref = p.numerics == 0;
    const bool bf = p.io_dtype == kBF16;

    for (int i = tid; i < K * VT; i += kSimtThreads) {
        const int r = i / VT, c = i % VT;
        float x = 0.0f;
        if (p.h0 && c < vcount) x = load_io(p.h0, p.h0_dtype, n * p.h0_sn + hv * p.h0_sh + r * p.h0_sk + (v0 + c) * p.h0_sv);
        S[i] = ref ? round_bf16(x) : x;
    }
    const int64_t nchunks = (si.len + kChunk - 1) / kChunk;
    const int trow = tid >> 2;                // token row of the MMA1/epi1 mapping
    const int j0 = (tid & 3) * (VT / 4);      // first of this thread's 8 columns

    for (int64_t c = 0; c < nchunks; ++c) {
        const int64_t t0 = si.bos + c * kChunk;
        const int len = static_cast<int>(si.len - c * kChunk < kChunk ? si.len - c * kChunk : kChunk);
        __syncthreads();
        // h[:, chunk] = state before the chunk (generate_golden.py:400)
        const int64_t hbase = si.b * p.h_sb + (si.boh + c) * p.h_sc + hv * p.h_sh + v0;
        for (int i = tid; i < K * VT; i += kSimtThreads) {
            const int r = i / VT, cc = i % VT;
            const float s = S[i];
            if (cc < vcount) store_io(p.h, p.io_dtype, hbase + r * p.h_sk + cc, s);
            Sb[i] = (bf && !ref) ? round_bf16(s) : s;
        }
        for (int i = tid; i < 64 * K; i += kSimtThreads) {
            const int t = i / K, kk = i % K;
            float wv = 0.0f, kv = 0.0f;
            if (t < len) {
                wv = load_io(p.w, p.io_dtype, si.b * p.w_sb + (t0 + t) * p.w_st + hv * p.w_sh + kk);
                kv = load_io(p.k, p.io_dtype, si.b * p.k_sb + (t0 + t) * p.k_st + kh * p.k_sh + kk);
            }
            Wc[t * (K + 1) + kk] = wv;
            Kc[t * (K + 1) + kk] = kv;
        }
        if (tid < 64) {
            const int64_t gb = si.b * p.g_sb + hv * p.g_sh;
            float gt = 1.0f;
            if (tid < len) {
                if (ref) {
                    const float gl = p.g[gb + (t0 + len - 1) * p.g_st];
                    gt = ref_gate(gl, p.g[gb + (t0 + tid) * p.g_st]);
                } else if (p.use_g) {
                    const float gl = p.g[gb + (t0 + len - 1) * p.g_st];
                    gt = safe_exp(gl - p.g[gb + (t0 + tid) * p.g_st]);
                }
            }
            gate[tid] = gt;
            if (tid == 0) {
                float a = 1.0f;
                if (ref)
                    a = ref_alpha(p.g[gb + (t0 + len - 1) * p.g_st]);
                else if (p.use_g)
                    a = expf(p.g[gb + (t0 + len - 1) * p.g_st]);
                s_alpha = a;
            }
        }
        __syncthreads();

        // MMA1 + epilogue 1: v_new = u - w . S, v_decay = v_new * gate.
        {
            float acc[VT / 4];
#pragma unroll
            for (int j = 0; j < VT / 4; ++j) acc[j] = 0.0f;
            for (int kk = 0; kk < K; ++kk) {
                const float a = Wc[trow * (K + 1) + kk];
#pragma unroll
                for (int j = 0; j < VT / 4; ++j) acc[j] = fmaf(a, Sb[kk * VT + j0 + j], acc[j]);
            }
            const float gt = gate[trow];
#pragma unroll
            for (int j = 0; j < VT / 4; ++j) {
                const int col = j0 + j;
                const bool valid = trow < len && col < vcount;
                float vd = 0.0f;
                if (valid) {
                    const int64_t ui = si.b * p.u_sb + (t0 + trow) * p.u_st + hv * p.u_sh + v0 + col;
                    const float uu = load_io(p.u, p.io_dtype, ui);
                    float vn;
                    if (ref) {
                        vn = ref_vnew(uu, acc[j]);
                        vd = ref_vdecay(vn, gt);
                    } else {
                        vn = uu - acc[j];
                        vd = vn * gt;
                        if (bf) vd = round_bf16(vd);
                    }
                    if (p.v_new)
                        store_io(p.v_new, p.io_dtype, si.b * p.v_sb + (t0 + trow) * p.v_st + hv * p.v_sh + v0 + col,
                                 vn);
                }
                Vd[trow * VT + col] = vd;
            }
        }
        __syncthreads();

        // MMA2 + epilogue 2: S = decay(S) + k^T . v_decay.
        const float alpha = s_alpha;
        for (int r = trow; r < K; r += 64) {
            float acc[VT / 4];
#pragma unroll
            for (int j = 0; j < VT / 4; ++j) acc[j] = 0.0f;
            for (int t = 0; t < 64; ++t) {
                const float a = Kc[t * (K + 1) + r];
#pragma unroll
                for (int j = 0; j < VT / 4; ++j) acc[j] = fmaf(a, Vd[t * VT + j0 + j], acc[j]);
            }
#pragma unroll
            for (int j = 0; j < VT / 4; ++j) {
                float& s = S[r * VT + j0 + j];
                s = ref ? ref_state(s, alpha, acc[j]) : fmaf(s, alpha, acc[j]);
            }
        }
    }
    __syncthreads();
    if (p.final_state) {
        for (int i = tid; i < K * VT; i += kSimtThreads) {
            const int r = i / VT, cc = i % VT;
            if (cc < vcount) store_io(p.final_state, p.f_dtype, n * p.f_sn + hv * p.f_sh + r * p.f_sk + (v0 + cc) * p.f_sv, S[i]);
        }
    }
}

// Varlen metadata (one block): validates cu_seqlens, writes each sequence's
// first chunk index (the reference's serial prefix over cu_seqlens,
// op_kernel/chunk_gated_delta_rule_fwd_h.h:308-327, done once instead of per
// task) and, for up to 1024 sequences, a longest-first launch order.
__global__ void __launch_bounds__(1024) varlen_prep_kernel(const int64_t* cu, int64_t N, int64_t T, int64_t NT,
                                                          int32_t* chunk_base, int32_t* order, int* status)
{
    __shared__ long long s_part[1024];
    __shared__ int s_bad;
    const int tid = threadIdx.x;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    const int64_t per = (N + blockDim.x - 1) / blockDim.x;
    const int64_t lo = tid * per, hi = (lo + per < N ? lo + per : N);
    long long sum = 0;
    for (int64_t i = lo; i < hi; ++i) {
        const int64_t L = cu[i + 1] - cu[i];
        if (L < 0) s_bad = 1;
        sum += (L + kChunk - 1) / kChunk;
    }
    s_part[tid] = sum;
    __syncthreads();
    if (tid == 0) {
        long long run = 0;
        for (int i = 0; i < (int)blockDim.x; ++i) {
            const long long v = s_part[i];
            s_part[i] = run;
            run += v;
        }
        // h must have a slot for every chunk (a caller may size it for more)
        if (cu[0] != 0 || cu[N] != T || run > NT) s_bad = 1;
    }
    __syncthreads();
    long long run = s_part[tid];
    for (int64_t i = lo; i < hi; ++i) {
        chunk_base[i] = static_cast<int32_t>(run);
        run += (cu[i + 1] - cu[i] + kChunk - 1) / kChunk;
    }
    if (tid == 0) chunk_base[N] = static_cast<int32_t>(NT);
    // Longest first: rank of sequence i = #sequences with more chunks, ties by index.
    if (N <= 1024) {
        for (int64_t i = tid; i < N; i += blockDim.x) {
            const int64_t li = cu[i + 1] - cu[i];
            int64_t r = 0;
            for (int64_t j = 0; j < N; ++j) {
                const int64_t lj = cu[j + 1] - cu[j];
                r += (lj > li) || (lj == li && j < i);
            }
            order[r] = static_cast<int32_t>(i);
        }
    } else {
        for (int64_t i = tid; i < N; i += blockDim.x) order[i] = static_cast<int32_t>(i);
    }
    __syncthreads();
    if (tid == 0 && s_bad && status) atomicOr(status, 0x2);
}

}  // namespace cgdr
