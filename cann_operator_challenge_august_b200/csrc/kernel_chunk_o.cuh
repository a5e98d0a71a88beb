// Chunk output of Gated DeltaNet prefill on tcgen05 (sm_100a): the consumer
// of the hidden-state recurrence's outputs h and v_new.
//
// For one 64-token chunk c of one sequence, value head hv and V tile (a "tile"):
//   S    = q . k^T                                      (64 x 64)
//   P    = bf16(bf16(S) * scale * exp(g_i - g_j))       for j <= i, else 0
//   o    = bf16((q . h[c]) * scale * exp(g_i) + P . v_new)   (64 x VT)
// which is the reference's stage-2 inter-chunk term plus its stage 3
// (ref/chunk_gated_delta_rule/tests/pytest/chunk_gated_delta_rule_benchmark.py:77-79
// and :129 for the inter-chunk term, :145-175 for the masked intra-chunk term;
// the NPU kernel op_kernel/arch22/chunk_gated_delta_rule_stage3.h:131-168
// rounds P the same way).  The reference rounds q * scale * exp(g) to bf16
// before its product with h; here q . h is scaled per row in fp32 (the
// arithmetic of the fla chunk_fwd_o kernel), and the two products accumulate
// in one fp32 TMEM accumulator rounded to bf16 once.
//
// Tiles are independent and the op is HBM-bound (~96 KB in and 16 KB out per
// tile at K = V = 128), so the kernel is persistent: one CTA per SM walks the
// tiles blockIdx.x, blockIdx.x + gridDim.x, ... and keeps the next tile's
// loads in flight while the current one computes.
//
// Warp roles (320 threads):
//   warp 0     TMA producer: q, k, v_new, h of a tile into a STAGES-deep ring;
//              the 64 gate values by cp.async;
//   warp 1     MMA issuer and TMEM owner (512 columns: two accumulator sets
//              of O [64 x VT] at +0 and S [64 x 64] at +128, 256 apart);
//   warps 2-9  epilogue: warp w reads TMEM lanes 32(w%4).. (rows 16(w%4)..+15
//              of an M=64 accumulator) and half of the columns ((w-2)/4).
//
// Per tile i (stage s, accumulator set a = i % 2):
//   MMA    S[a]  = q . k^T ; O[a] = q . h       M=64 N=64 / VT, K=K
//   epi A  P from S[a] in place of k (read by MMA_S only); O[a] rows scaled by
//          scale * exp(g_i) in TMEM (tcgen05.ld / st)
//   MMA    O[a] += P . v_new                    M=64 N=VT K=64   (B MN-major)
//   epi B  o = bf16(O[a]) -> swizzled staging tile -> coalesced 16-byte stores
// The epilogue runs A(i) before B(i-1), so tile i-1's output products run on
// the tensor cores while tile i's P is formed.
//
// Every wait is bounded; on expiry the CTA records the role in the status
// word, drains its own copies and MMAs, and returns.  The epilogue warps never
// leave their loop early, so their named barriers always see all four.
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
    int64_t n_tiles;         // rows * H * n_vtiles
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
};

struct ChunkOArgs {
    ChunkOMaps maps;
    ChunkOParams p;
};

template <int K_, int VT, int STAGES>
struct ChunkOConfig {
    static_assert(K_ == 64 || K_ == 128, "chunk output: K in {64, 128}");
    static_assert(VT == 64 || VT == 128, "chunk output: V tile in {64, 128}");
    static constexpr int kEpiWarps = 8;
    static constexpr int kEpiThreads = 32 * kEpiWarps;
    static constexpr int kThreads = 64 + kEpiThreads;
    static constexpr int kSubK = K_ / 64;
    static constexpr int kSubV = VT / 64;
    static constexpr int kTileK = K_ * 128;    // [64 tokens][K] bf16 (q or k)
    static constexpr int kTileV = VT * 128;    // [64 tokens][VT] bf16
    static constexpr int kHSub = K_ * 128;     // [K rows][64 cols] bf16 sub-tile of h
    static constexpr int kOffQ = 0;            // offsets within a stage
    static constexpr int kOffK = kTileK;       // P [64][64] replaces k after MMA_S
    static constexpr int kOffV = 2 * kTileK;
    static constexpr int kOffH = 2 * kTileK + kTileV;
    static constexpr int kStageBytes = kOffH + kSubV * kHSub;
    static constexpr int kOffG = STAGES * kStageBytes;                        // [STAGES][64] fp32
    static constexpr int kOffOut = (kOffG + STAGES * 256 + 1023) / 1024 * 1024;  // o staging tile
    static constexpr int kOutBytes = VT * 128;
    static constexpr int kOffBar = kOffOut + kOutBytes;
    static constexpr int kNumBars = 2 * STAGES + 11;
    static constexpr int kUsed = kOffBar + kNumBars * 8 + 16;
    // more than half of an SM's shared memory: one CTA per SM, so the CTA's
    // 512 TMEM columns never wait for another CTA's
    static constexpr int kSmemBytes = (kUsed + 1024 > 120 * 1024) ? kUsed + 1024 : 120 * 1024;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kAccStride = 256;
    static constexpr uint32_t kTmemS = 128;
    static constexpr uint32_t kTx = kStageBytes;
    static constexpr uint32_t kIdescS = umma_idesc_bf16(64, 64, false, false);
    static constexpr uint32_t kIdescO = umma_idesc_bf16(64, VT, false, true);
};

struct ChunkOTile {
    int64_t b, t0, len, hrow, hv, kh;
    int v0;
    bool ok;
    bool pad;  // chunk_indices row (-1, -1): a padding row, skipped without a flag
};

__device__ __forceinline__ ChunkOTile chunk_o_tile(const ChunkOParams& p, int64_t tile, int vt_width)
{
    ChunkOTile t;
    const int vt = static_cast<int>(tile % p.n_vtiles);
    tile /= p.n_vtiles;
    t.hv = tile % p.H;
    const int64_t row = tile / p.H;
    t.kh = t.hv / (p.H / p.HK);
    t.v0 = vt * vt_width;
    t.ok = true;
    t.pad = false;
    if (p.varlen) {
        const int64_t n = p.chunk_indices[2 * row];
        const int64_t c = p.chunk_indices[2 * row + 1];
        t.pad = n == -1 && c == -1;
        t.ok = n >= 0 && n < p.N && c >= 0;
        int64_t bos = 0, eos = 0;
        if (t.ok) {
            bos = p.cu_seqlens[n];
            eos = p.cu_seqlens[n + 1];
            t.ok = bos >= 0 && eos <= p.T && bos + c * kChunk < eos;
        }
        t.b = 0;
        t.t0 = bos + c * kChunk;
        t.len = t.ok ? (eos - t.t0 < kChunk ? eos - t.t0 : kChunk) : 0;
        t.hrow = row;
    } else {
        t.b = row / p.nt_per_seq;
        const int64_t c = row % p.nt_per_seq;
        t.t0 = c * kChunk;
        t.len = p.T - t.t0 < kChunk ? p.T - t.t0 : kChunk;
        t.hrow = c;
    }
    return t;
}

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int K_, int VT, int STAGES>
__global__ void __launch_bounds__(320, 1) chunk_o_tc_kernel(const __grid_constant__ ChunkOArgs args)
{
    using Cfg = ChunkOConfig<K_, VT, STAGES>;
    const ChunkOParams& p = args.p;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* s_full = bars + 2 * STAGES;     // [2]
    uint64_t* p_ready = s_full + 2;           // [2]
    uint64_t* o_full = s_full + 4;            // [2]
    uint64_t* acc_empty = s_full + 6;         // [2]
    uint64_t* o1_full = s_full + 8;           // [2]  q . h done
    uint64_t* mma_drain = s_full + 10;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* never_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1 + 32);  // TMA bytes + 32 cp.async arrivals (gate values)
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&s_full[a], 1);
            mbar_init(&p_ready[a], Cfg::kEpiWarps);
            mbar_init(&o_full[a], 1);
            mbar_init(&acc_empty[a], Cfg::kEpiWarps);
            mbar_init(&o1_full[a], 1);
        }
        mbar_init(mma_drain, 1);
        *abort_flag = 0;
        *never_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&args.maps.q);
        prefetch_tensormap(&args.maps.k);
        prefetch_tensormap(&args.maps.v);
        prefetch_tensormap(&args.maps.h);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const WaitCtl ctl{abort_flag, p.status, p.timeout_ns};
    const uint32_t sbase = smem_u32(smem);
    float* gbase = reinterpret_cast<float*>(smem + Cfg::kOffG);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        int64_t it = 0;
        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const ChunkOTile t = chunk_o_tile(p, tile, VT);
            if (!t.ok) {
                if (lane == 0 && p.status && !t.pad) atomicOr(p.status, 0x2);
                continue;
            }
            const int s = static_cast<int>(it % STAGES);
            const uint32_t use = static_cast<uint32_t>(it / STAGES);
            bool go = true;
            if (it >= STAGES && lane == 0) go = mbar_wait(&empty[s], (use - 1) & 1, ctl, 0x10);
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (!go) break;
            uint8_t* st = smem + s * Cfg::kStageBytes;
            if (lane == 0) {
                const int ib = static_cast<int>(t.b), it0 = static_cast<int>(t.t0);
                mbar_arrive_expect_tx(&full[s], Cfg::kTx);
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubK; ++sub) {
                    tma_load_4d(&args.maps.q, st + Cfg::kOffQ + sub * 8192, &full[s], sub * 64,
                                static_cast<int>(t.kh), it0, ib);
                    tma_load_4d(&args.maps.k, st + Cfg::kOffK + sub * 8192, &full[s], sub * 64,
                                static_cast<int>(t.kh), it0, ib);
                }
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubV; ++sub) {
                    tma_load_4d(&args.maps.v, st + Cfg::kOffV + sub * 8192, &full[s], t.v0 + sub * 64,
                                static_cast<int>(t.hv), it0, ib);
                    tma_load_5d(&args.maps.h, st + Cfg::kOffH + sub * Cfg::kHSub, &full[s], t.v0 + sub * 64, 0,
                                static_cast<int>(t.hv), static_cast<int>(t.hrow), ib);
                }
            }
            if (p.g) {
                float* gs = gbase + 64 * s;
                const int64_t gb = t.b * p.g_sb + t.hv * p.g_sh;
                if (lane < t.len) cp_async_4(gs + lane, p.g + gb + (t.t0 + lane) * p.g_st);
                if (lane + 32 < t.len) cp_async_4(gs + lane + 32, p.g + gb + (t.t0 + lane + 32) * p.g_st);
            }
            cp_async_arrive_noinc(&full[s]);
            ++it;
        }
        // never leave while a load may still land in this CTA's shared memory
        if (lane == 0) {
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            const int64_t first = it > STAGES ? it - STAGES : 0;
            for (int64_t j = first; j < it; ++j)
                mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1, drain, 0x10);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs the loop; one elected lane issues the MMAs and commits.
        auto wait_warp = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, ctl, 0x20) ? 1 : 0) != 0;
        };
        int64_t it = 0;
        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const ChunkOTile t = chunk_o_tile(p, tile, VT);
            if (!t.ok) continue;
            const int s = static_cast<int>(it % STAGES);
            const int a = static_cast<int>(it & 1);
            const uint32_t st = sbase + s * Cfg::kStageBytes;
            const uint32_t acc = tmem + a * Cfg::kAccStride;
            if (!wait_warp(&full[s], static_cast<uint32_t>(it / STAGES) & 1)) break;
            if (it >= 2 && !wait_warp(&acc_empty[a], static_cast<uint32_t>(it / 2 - 1) & 1)) break;
            tc_fence_after();
            {
                const uint64_t da = umma_desc_sw128(st + Cfg::kOffQ, 16, 1024);
                const uint64_t db = umma_desc_sw128(st + Cfg::kOffK, 16, 1024);
                const uint64_t dh = umma_desc_sw128(st + Cfg::kOffH, Cfg::kHSub, 1024);
                if (elect_one_sync()) {
#pragma unroll
                    for (int kk = 0; kk < K_ / 16; ++kk) {
                        const uint64_t off = static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
                        tc_mma_bf16(acc + Cfg::kTmemS, da + off, db + off, Cfg::kIdescS, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&s_full[a]);
#pragma unroll
                    for (int kk = 0; kk < K_ / 16; ++kk)
                        tc_mma_bf16(acc, da + static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4),
                                    dh + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescO, kk > 0 ? 1u : 0u);
                    tc_commit(&o1_full[a]);
                }
                __syncwarp();
            }
            if (!wait_warp(&p_ready[a], static_cast<uint32_t>(it / 2) & 1)) break;
            tc_fence_after();
            {
                const uint64_t pa = umma_desc_sw128(st + Cfg::kOffK, 16, 1024);
                const uint64_t vb = umma_desc_sw128(st + Cfg::kOffV, 8192, 1024);
                if (elect_one_sync()) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_bf16(acc, pa + static_cast<uint64_t>((kk * 32) >> 4),
                                    vb + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescO, 1u);
                    tc_commit(&o_full[a]);
                    tc_commit(&empty[s]);
                }
                __syncwarp();
            }
            ++it;
        }
        if (elect_one_sync()) tc_commit(mma_drain);
        __syncwarp();
        WaitCtl drain{never_flag, p.status, p.timeout_ns};
        mbar_wait(mma_drain, 0, drain, 0x20);
    } else {
        // ------------------------------------------------------------ epilogue
        const int et = threadIdx.x - 64;     // 0..255
        const int qd = warp & 3;             // TMEM lane quadrant of this warp
        const int ch = (warp - 2) >> 2;      // column half of this warp
        const int ra = 16 * qd + (lane >> 2);
        const int rb = ra + 8;
        const int pc = 2 * (lane & 3);
        const float sc = p.scale;
        constexpr int kOCols = VT / 2;       // O columns per warp
        uint8_t* stg = smem + Cfg::kOffOut;
        bool ok = true;
        int64_t it = 0;
        ChunkOTile prev{};

        // o of the tile with index j (accumulator set j % 2)
        auto output = [&](int64_t j, const ChunkOTile& t) {
            const int a = static_cast<int>(j & 1);
            const uint32_t acc = tmem + a * Cfg::kAccStride;
            if (ok) ok = mbar_wait(&o_full[a], static_cast<uint32_t>(j / 2) & 1, ctl, 0x40);
            ok = __all_sync(0xffffffffu, ok) != 0;
            uint32_t r[kOCols / 32][16];
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int cb = 0; cb < kOCols / 32; ++cb)
                    tmem_ld_16x256b_x4(acc + ((32u * qd) << 16) + static_cast<uint32_t>(kOCols * ch + 32 * cb), r[cb]);
                tmem_wait_ld();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
            // the staging tile is free once every thread stored the previous tile's rows
            epi_bar_sync();
            if (ok) {
#pragma unroll
                for (int cb = 0; cb < kOCols / 32; ++cb)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                        for (int half = 0; half < 2; ++half) {
                            const int i = half ? rb : ra;
                            const int col = kOCols * ch + 32 * cb + 8 * jj + pc;
                            *reinterpret_cast<uint32_t*>(stg + sw128_off(i, col, 8192)) =
                                pack_bf16x2(__uint_as_float(r[cb][4 * jj + 2 * half]),
                                            __uint_as_float(r[cb][4 * jj + 2 * half + 1]));
                        }
            }
            epi_bar_sync();
            if (ok) {
                // 16-byte chunks, consecutive threads along a row: each warp writes whole rows
                constexpr int kChunksPerRow = VT / 8;
                __nv_bfloat16* orow = p.o + t.b * p.o_sb + t.t0 * p.o_st + t.hv * p.o_sh + t.v0;
#pragma unroll
                for (int e = et; e < 64 * kChunksPerRow; e += Cfg::kEpiThreads) {
                    const int row = e / kChunksPerRow, cc = e % kChunksPerRow;
                    if (row < t.len)
                        *reinterpret_cast<uint4*>(orow + row * p.o_st + 8 * cc) =
                            *reinterpret_cast<const uint4*>(stg + sw128_off(row, 8 * cc, 8192));
                }
            }
        };

        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const ChunkOTile t = chunk_o_tile(p, tile, VT);
            if (!t.ok) continue;
            const int s = static_cast<int>(it % STAGES);
            const int a = static_cast<int>(it & 1);
            uint8_t* st = smem + s * Cfg::kStageBytes;
            const float* gs = gbase + 64 * s;
            // ---- A(it): P and the row scaling of q . h
            if (ok) ok = mbar_wait(&full[s], static_cast<uint32_t>(it / STAGES) & 1, ctl, 0x40);
            if (ok) ok = mbar_wait(&s_full[a], static_cast<uint32_t>(it / 2) & 1, ctl, 0x40);
            ok = __all_sync(0xffffffffu, ok) != 0;
            if (ok) {
                tc_fence_after();
                // S (this warp's 32 columns)
                uint32_t sr[16];
                const uint32_t acc = tmem + a * Cfg::kAccStride;
                tmem_ld_16x256b_x4(acc + ((32u * qd) << 16) + Cfg::kTmemS + 32 * ch, sr);
                tmem_wait_ld();
                const float ga = (p.g && ra < t.len) ? gs[ra] : 0.0f;
                const float gb = (p.g && rb < t.len) ? gs[rb] : 0.0f;
                uint8_t* pt = st + Cfg::kOffK;
                // the decay factors use the fast exp intrinsic: P is rounded to bf16
                // (8 significant bits), far coarser than the intrinsic's error
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int j = 32 * ch + 8 * jj + pc;
                    const float gj0 = (p.g && j < t.len) ? gs[j] : 0.0f;
                    const float gj1 = (p.g && j + 1 < t.len) ? gs[j + 1] : 0.0f;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int i = half ? rb : ra;
                        const float gi = half ? gb : ga;
                        const float s0 = round_bf16(__uint_as_float(sr[4 * jj + 2 * half]));
                        const float s1 = round_bf16(__uint_as_float(sr[4 * jj + 2 * half + 1]));
                        const float x0 = (j <= i) ? __fmul_rn(__fmul_rn(s0, sc), __expf(gi - gj0)) : 0.0f;
                        const float x1 = (j + 1 <= i) ? __fmul_rn(__fmul_rn(s1, sc), __expf(gi - gj1)) : 0.0f;
                        *reinterpret_cast<uint32_t*>(pt + sw128_off(i, j, 8192)) = pack_bf16x2(x0, x1);
                    }
                }
                if (t.len < kChunk) {
                    // v_new rows past the chunk's end belong to another sequence (or are
                    // fill): zero them so that no value of theirs reaches a product
                    const int rows = kChunk - static_cast<int>(t.len);
                    for (int e = et; e < Cfg::kSubV * rows * 8; e += Cfg::kEpiThreads) {
                        const int sub = e / (rows * 8), rr = static_cast<int>(t.len) + (e / 8) % rows, c8 = e & 7;
                        *reinterpret_cast<uint4*>(st + Cfg::kOffV + sub * 8192 + rr * 128 + c8 * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                }
                // O = q . h scaled per row by scale * exp(g_i), in TMEM
                ok = mbar_wait(&o1_full[a], static_cast<uint32_t>(it / 2) & 1, ctl, 0x40);
            }
            ok = __all_sync(0xffffffffu, ok) != 0;
            if (ok) {
                tc_fence_after();
                const uint32_t acc = tmem + a * Cfg::kAccStride + ((32u * qd) << 16) + static_cast<uint32_t>(kOCols * ch);
                uint32_t r[kOCols / 32][16];
#pragma unroll
                for (int cb = 0; cb < kOCols / 32; ++cb) tmem_ld_16x256b_x4(acc + 32 * cb, r[cb]);
                const float fa = __fmul_rn(sc, expf((p.g && ra < t.len) ? gs[ra] : 0.0f));
                const float fb = __fmul_rn(sc, expf((p.g && rb < t.len) ? gs[rb] : 0.0f));
                tmem_wait_ld();
#pragma unroll
                for (int cb = 0; cb < kOCols / 32; ++cb)
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        r[cb][e] = __float_as_uint(__fmul_rn(__uint_as_float(r[cb][e]), (e & 2) ? fb : fa));
#pragma unroll
                for (int cb = 0; cb < kOCols / 32; ++cb) tmem_st_16x256b_x4(acc + 32 * cb, r[cb]);
                tmem_wait_st();
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_ready[a]);
            // ---- B(it-1): the previous tile's output
            if (it >= 1) output(it - 1, prev);
            prev = t;
            ++it;
        }
        if (it >= 1) output(it - 1, prev);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace cgdr
