// Chunk output of Gated DeltaNet prefill on tcgen05 (sm_100a): the consumer
// of the hidden-state recurrence's outputs h and v_new.
//
// For one 64-token chunk c of one sequence, value head hv and V tile:
//   q'   = bf16(q * scale * exp(g))                     per row
//   S    = q . k^T                                      (64 x 64)
//   P    = bf16(bf16(S) * scale * exp(g_i - g_j))       for j <= i, else 0
//   o    = bf16(q' . h[c] + P . v_new)                  (64 x VT)
// which is the reference's stage-2 inter-chunk term plus its stage 3
// (ref/chunk_gated_delta_rule/tests/pytest/chunk_gated_delta_rule_benchmark.py:77-79
// for q', :129 for q'.S, :145-175 for the masked intra-chunk term;
// the NPU kernel op_kernel/arch22/chunk_gated_delta_rule_stage3.h:131-168
// rounds P the same way).  The two products accumulate in one fp32 TMEM
// accumulator and are rounded to bf16 once.
//
// Chunks are independent, so one CTA owns one (chunk, head, V tile) and the
// grid covers them all; two CTAs share an SM so one's loads overlap the
// other's tensor-core work.  128 threads: thread 0 issues the TMA loads and
// the MMAs, all four warps run the element-wise phases (warp w reads TMEM
// lanes 32w..32w+15, which hold rows 16w..16w+15 of an M=64 accumulator).
//
//   MMA_S  S[i,j]  = sum_k q[i,k] k[j,k]        M=64 N=64 K=K   (A, B K-major)
//   MMA_O  O[i,v]  = sum_k q'[i,k] h[k,v]       M=64 N=VT K=K   (A K-major, B MN-major)
//   MMA_PV O[i,v] += sum_j P[i,j] v_new[j,v]    M=64 N=VT K=64  (A K-major, B MN-major)
//
// Every wait is bounded; on expiry the CTA records the role in the status
// word, drains its own copies and MMAs, and returns.
#pragma once

#include "common.cuh"
#include "kernel_tc.cuh"
#include "ptx.cuh"

namespace cgdr {

struct ChunkOParams {
    const float* g;          // [B, T, H] chunk-local cumulative log gate (nullptr: no gate)
    __nv_bfloat16* o;        // [B, T, H, V]
    const int64_t* cu_seqlens;      // [N + 1] (varlen) or nullptr
    const int64_t* chunk_indices;   // [NT, 2] (varlen) or nullptr
    int64_t B, T, H, HK, K, V, N, NT;
    int64_t nt_per_seq;      // fixed length: chunks per batch row
    int64_t g_sb, g_st, g_sh;
    int64_t o_sb, o_st, o_sh;
    int32_t n_vtiles;
    int32_t varlen;
    float scale;
    int* status;
    uint64_t timeout_ns;
};

struct ChunkOMaps {
    CUtensorMap q;  // dims (K, HK, T, B), box (64, 1, 64, 1)
    CUtensorMap k;  // dims (K, HK, T, B), box (64, 1, 64, 1)
    CUtensorMap v;  // dims (V, H, T, B),  box (64, 1, 64, 1)   v_new
    CUtensorMap h;  // dims (V, K, H, NT, B), box (64, K, 1, 1, 1)
    CUtensorMap o;  // dims (V, H, T, B),  box (64, 1, 64, 1)   store
};

struct ChunkOArgs {
    ChunkOMaps maps;
    ChunkOParams p;
};

template <int K_, int VT>
struct ChunkOConfig {
    static_assert(K_ == 64 || K_ == 128, "chunk output: K in {64, 128}");
    static_assert(VT == 64 || VT == 128, "chunk output: V tile in {64, 128}");
    static constexpr int kThreads = 128;
    static constexpr int kSubK = K_ / 64;
    static constexpr int kSubV = VT / 64;
    static constexpr int kTileKBytes = K_ * 128;   // [64 tokens][K] bf16
    static constexpr int kHSubBytes = K_ * 128;    // [K rows][64 cols] bf16
    static constexpr int kOffQ = 0;
    static constexpr int kOffQP = kOffQ + kTileKBytes;
    static constexpr int kOffK = kOffQP + kTileKBytes;       // P [64][64] reuses it after MMA_S
    static constexpr int kOffV = kOffK + kTileKBytes;
    static constexpr int kOffH = kOffV + VT * 128;
    static constexpr int kOffG = kOffH + kSubV * kHSubBytes;  // 64 fp32
    static constexpr int kOffBar = kOffG + 64 * 4;
    static constexpr int kNumBars = 5;
    static constexpr int kUsed = kOffBar + kNumBars * 8 + 16;
    // o staging reuses q and q' (both free once MMA_PV completed)
    static_assert(2 * kTileKBytes >= VT * 128, "o staging must fit in the q and q' tiles");
    // At most two CTAs per SM: two 256-column TMEM allocations fill the 512 columns.
    static constexpr int kSmemBytes = (kUsed + 1024 > 80 * 1024) ? kUsed + 1024 : 80 * 1024;
    static constexpr uint32_t kTmemCols = 256;  // O at [0, VT), S at [128, 192)
    static constexpr uint32_t kTmemS = 128;
    static constexpr uint32_t kTxQK = 2 * kTileKBytes;
    static constexpr uint32_t kTxVH = VT * 128 + kSubV * kHSubBytes;
    static constexpr uint32_t kIdescS = umma_idesc_bf16(64, 64, false, false);
    static constexpr uint32_t kIdescO = umma_idesc_bf16(64, VT, false, true);
};

template <int K_, int VT>
__global__ void __launch_bounds__(128, 2) chunk_o_tc_kernel(const __grid_constant__ ChunkOArgs args)
{
    using Cfg = ChunkOConfig<K_, VT>;
    const ChunkOParams& p = args.p;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* bar_qk = bars;
    uint64_t* bar_vh = bars + 1;
    uint64_t* bar_s = bars + 2;
    uint64_t* bar_o = bars + 3;
    uint64_t* bar_drain = bars + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* never_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
    float* gs = reinterpret_cast<float*>(smem + Cfg::kOffG);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    // ---- which chunk: blockIdx.x = (row * H + hv) * n_vtiles + vt
    int64_t bid = blockIdx.x;
    const int vt = static_cast<int>(bid % p.n_vtiles);
    bid /= p.n_vtiles;
    const int64_t hv = bid % p.H;
    const int64_t row = bid / p.H;
    int64_t b, t0, len, hrow;
    if (p.varlen) {
        const int64_t n = p.chunk_indices[2 * row];
        const int64_t c = p.chunk_indices[2 * row + 1];
        bool bad = n < 0 || n >= p.N || c < 0;
        int64_t bos = 0, eos = 0;
        if (!bad) {
            bos = p.cu_seqlens[n];
            eos = p.cu_seqlens[n + 1];
            bad = bos < 0 || eos > p.T || bos + c * kChunk >= eos;
        }
        if (bad) {
            if (tid == 0 && p.status) atomicOr(p.status, 0x2);
            return;
        }
        b = 0;
        t0 = bos + c * kChunk;
        len = eos - t0 < kChunk ? eos - t0 : kChunk;
        hrow = row;
    } else {
        b = row / p.nt_per_seq;
        const int64_t c = row % p.nt_per_seq;
        t0 = c * kChunk;
        len = p.T - t0 < kChunk ? p.T - t0 : kChunk;
        hrow = c;
    }
    const int64_t kh = hv / (p.H / p.HK);
    const int v0 = vt * VT;
    const bool partial = len < kChunk;

    if (tid == 0) {
        mbar_init(bar_qk, 1);
        mbar_init(bar_vh, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        *never_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    // gate inputs (rows past the chunk's end read as 0: exp(0) keeps them finite)
    if (tid < kChunk) {
        float x = 0.0f;
        if (p.g && tid < len) x = p.g[b * p.g_sb + (t0 + tid) * p.g_st + hv * p.g_sh];
        gs[tid] = x;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const WaitCtl ctl{abort_flag, p.status, p.timeout_ns};
    const uint32_t sbase = smem_u32(smem);
    uint8_t* q_t = smem + Cfg::kOffQ;
    uint8_t* qp_t = smem + Cfg::kOffQP;
    uint8_t* p_t = smem + Cfg::kOffK;
    uint8_t* v_t = smem + Cfg::kOffV;

    // ---- loads
    if (tid == 0) {
        const int ib = static_cast<int>(b), it = static_cast<int>(t0);
        mbar_arrive_expect_tx(bar_qk, Cfg::kTxQK);
#pragma unroll
        for (int sub = 0; sub < Cfg::kSubK; ++sub) {
            tma_load_4d(&args.maps.q, smem + Cfg::kOffQ + sub * 8192, bar_qk, sub * 64, static_cast<int>(kh), it, ib);
            tma_load_4d(&args.maps.k, smem + Cfg::kOffK + sub * 8192, bar_qk, sub * 64, static_cast<int>(kh), it, ib);
        }
        mbar_arrive_expect_tx(bar_vh, Cfg::kTxVH);
#pragma unroll
        for (int sub = 0; sub < Cfg::kSubV; ++sub) {
            tma_load_4d(&args.maps.v, smem + Cfg::kOffV + sub * 8192, bar_vh, v0 + sub * 64, static_cast<int>(hv), it,
                        ib);
            tma_load_5d(&args.maps.h, smem + Cfg::kOffH + sub * Cfg::kHSubBytes, bar_vh, v0 + sub * 64, 0,
                        static_cast<int>(hv), static_cast<int>(hrow), ib);
        }
        // MMA_S as soon as q and k landed
        if (mbar_wait(bar_qk, 0, ctl, 0x20)) {
            tc_fence_after();
            const uint64_t a = umma_desc_sw128(sbase + Cfg::kOffQ, 16, 1024);
            const uint64_t bdesc = umma_desc_sw128(sbase + Cfg::kOffK, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < K_ / 16; ++kk) {
                const uint64_t off = static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
                tc_mma_bf16(tmem + Cfg::kTmemS, a + off, bdesc + off, Cfg::kIdescS, kk > 0 ? 1u : 0u);
            }
            tc_commit(bar_s);
        }
    }

    // ---- q' = bf16(q * scale * exp(g)): thread t scales half a row in place of
    // the swizzle (the 16-byte chunks of a row stay within the row's 128 bytes)
    bool ok = mbar_wait(bar_qk, 0, ctl, 0x40);
    if (ok) {
        constexpr int kChunksPerThread = K_ * 2 / 16 / 2;  // 16-byte chunks per half row
        const int r = tid >> 1, half = tid & 1;
        const float f = p.scale;
        const float eg = expf(gs[r]);
#pragma unroll
        for (int i = 0; i < kChunksPerThread; ++i) {
            // chunk index within the row: K=128 -> sub-tile `half`, 8 chunks; K=64 -> chunks 4*half + i
            const int idx = half * kChunksPerThread + i;
            const uint32_t off = (idx >> 3) * 8192 + r * 128 + (idx & 7) * 16;
            const uint4 x = *reinterpret_cast<const uint4*>(q_t + off);
            uint4 y;
            const uint32_t* xs = &x.x;
            uint32_t* ys = &y.x;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 v = unpack_bf16x2(xs[j]);
                ys[j] = pack_bf16x2(__fmul_rn(__fmul_rn(v.x, f), eg), __fmul_rn(__fmul_rn(v.y, f), eg));
            }
            *reinterpret_cast<uint4*>(qp_t + off) = y;
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && ok && !*abort_flag) {
        // MMA_O = q' . h once v_new and h landed
        if (mbar_wait(bar_vh, 0, ctl, 0x20)) {
            tc_fence_after();
            const uint64_t a = umma_desc_sw128(sbase + Cfg::kOffQP, 16, 1024);
            const uint64_t bdesc = umma_desc_sw128(sbase + Cfg::kOffH, Cfg::kHSubBytes, 1024);
#pragma unroll
            for (int kk = 0; kk < K_ / 16; ++kk)
                tc_mma_bf16(tmem, a + static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4),
                            bdesc + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescO, kk > 0 ? 1u : 0u);
        }
    }

    // ---- P from S (rows ra, rb; column pairs 8jj + 2(lane%4) of each 32-column block)
    const int ra = 16 * warp + (lane >> 2);
    const int rb = ra + 8;
    const int pc = 2 * (lane & 3);
    ok = ok && mbar_wait(bar_s, 0, ctl, 0x40);
    ok = __all_sync(0xffffffffu, ok) != 0;  // tcgen05.ld is warp-collective
    if (ok) {
        tc_fence_after();
        uint32_t sr[2][16];
        tmem_ld_16x256b_x4(tmem + ((32u * warp) << 16) + Cfg::kTmemS, sr[0]);
        tmem_ld_16x256b_x4(tmem + ((32u * warp) << 16) + Cfg::kTmemS + 32, sr[1]);
        tmem_wait_ld();
        const float ga = gs[ra], gb = gs[rb];
        const float sc = p.scale;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int i = half ? rb : ra;
                    const float gi = half ? gb : ga;
                    const int j = 32 * blk + 8 * jj + pc;
                    float x[2];
#pragma unroll
                    for (int bit = 0; bit < 2; ++bit) {
                        const float s = round_bf16(__uint_as_float(sr[blk][4 * jj + 2 * half + bit]));
                        const float d = expf(gi - gs[j + bit]);
                        x[bit] = (j + bit <= i) ? __fmul_rn(__fmul_rn(s, sc), d) : 0.0f;
                    }
                    *reinterpret_cast<uint32_t*>(p_t + sw128_off(i, j, 8192)) = pack_bf16x2(x[0], x[1]);
                }
        if (partial) {
            // rows of v_new past the chunk's end belong to another sequence (or are
            // fill): zero them so that no value of theirs reaches a product
            ok = mbar_wait(bar_vh, 0, ctl, 0x40);
            if (ok) {
                const int rows = kChunk - static_cast<int>(len);
                for (int e = tid; e < Cfg::kSubV * rows * 8; e += Cfg::kThreads) {
                    const int sub = e / (rows * 8), rr = static_cast<int>(len) + (e / 8) % rows, ch = e & 7;
                    *reinterpret_cast<uint4*>(v_t + sub * 8192 + rr * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
                }
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && ok && !*abort_flag) {
        const uint64_t a = umma_desc_sw128(sbase + Cfg::kOffK, 16, 1024);
        const uint64_t bdesc = umma_desc_sw128(sbase + Cfg::kOffV, 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
            tc_mma_bf16(tmem, a + static_cast<uint64_t>((kk * 32) >> 4), bdesc + static_cast<uint64_t>((kk * 2048) >> 4),
                        Cfg::kIdescO, 1u);
        tc_commit(bar_o);
    }

    // ---- o = bf16(O)
    ok = ok && mbar_wait(bar_o, 0, ctl, 0x40);
    ok = __all_sync(0xffffffffu, ok) != 0;
    const bool plain_store = partial && p.varlen;
    if (ok) {
        tc_fence_after();
        uint8_t* o_t = smem + Cfg::kOffQ;  // staging over q and q'
#pragma unroll
        for (int cb = 0; cb < VT / 32; ++cb) {
            uint32_t r[16];
            tmem_ld_16x256b_x4(tmem + ((32u * warp) << 16) + static_cast<uint32_t>(32 * cb), r);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int i = half ? rb : ra;
                    const int col = 32 * cb + 8 * jj + pc;
                    const uint32_t v2 = pack_bf16x2(__uint_as_float(r[4 * jj + 2 * half]),
                                                    __uint_as_float(r[4 * jj + 2 * half + 1]));
                    if (plain_store) {
                        if (i < len)
                            *reinterpret_cast<uint32_t*>(p.o + b * p.o_sb + (t0 + i) * p.o_st + hv * p.o_sh + v0 +
                                                         col) = v2;
                    } else {
                        *reinterpret_cast<uint32_t*>(o_t + sw128_off(i, col, 8192)) = v2;
                    }
                }
        }
        if (!plain_store) {
            fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) {
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubV; ++sub)
                    tma_store_4d(&args.maps.o, o_t + sub * 8192, v0 + sub * 64, static_cast<int>(hv),
                                 static_cast<int>(t0), static_cast<int>(b));
                bulk_commit_group();
            }
        }
    }

    // ---- drain: loads landed, MMAs completed, the o store read its staging
    if (tid == 0) {
        WaitCtl drain{never_flag, p.status, p.timeout_ns};
        mbar_wait(bar_qk, 0, drain, 0x10);
        mbar_wait(bar_vh, 0, drain, 0x10);
        tc_commit(bar_drain);
        mbar_wait(bar_drain, 0, drain, 0x20);
        bulk_wait_group_read0();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace cgdr
