// WY representation of Gated DeltaNet prefill on sm_100a: the producer of the
// hidden-state recurrence's inputs w, u and the chunk-local cumulative gate.
//
// For one 64-token chunk of one sequence and value head (rows i, j, m of the
// chunk; the key head is hv / (H / HK)):
//   g_c  = cumsum of g within the chunk                      (fp64 scan, fp32 out)
//   A    = bf16(k k^T)[i, j] * beta_i * exp(g_c,i - g_c,j)   for j < i, else 0
//   T    = bf16((I + A)^-1)
//   w    = bf16(T . bf16(beta * exp(g_c) * k))              [64, K]
//   u    = bf16(T . bf16(beta * v))                          [64, V]
// the reference's stage 1 (ref/chunk_gated_delta_rule/tests/pytest/
// chunk_gated_delta_rule_benchmark.py:55-83; the reference keeps -w as
// "k_cumdecay", :74 and :82).  The inverse is restated from the mathematics
// of a unit lower-triangular matrix: forward substitution inside the four
// 16 x 16 diagonal blocks, then block forward substitution for the blocks
// below the diagonal, T_ij = -T_ii sum_{m=j}^{i-1} A_im T_mj, in fp32.
//
// Persistent kernel, one CTA per SM walking tiles (chunk row, value head)
// blockIdx.x, blockIdx.x + gridDim.x, ...  Warp roles (352 threads):
//   warp 0      TMA producer: k and v of a tile into a STAGES-deep ring;
//   warp 1      MMA issuer and TMEM owner (512 columns: two sets of W [64 x K]
//               at +0 and U [64 x V] at +128, 256 apart; k k^T is written into
//               W's first 64 columns and read before W's product overwrites it);
//   warp 2      gate loader: beta and g of the tile (plain loads), the fp64
//               cumulative sum, the g_c output, both into the stage;
//   warps 3-10  epilogue: warp w reads TMEM lanes 32(w%4).. (rows 16(w%4)..+15
//               of an M=64 accumulator) and half of the columns ((w-3)/4).
// Per tile (stage s, accumulator set a):
//   MMA   KK[a] = k k^T                       M=64 N=64 K=K (both K-major)
//   epi   A; k' = beta e^g k and v' = beta v in place; T; T -> bf16 tile T[a]
//   MMA   W[a] = T k' ; U[a] = T v'           M=64 N=K / V K=64 (B MN-major)
//   epi   w, u = bf16 -> swizzled staging -> coalesced 16-byte stores
// Every wait is bounded and no role leaves early (see kernel_chunk_o.cuh).
#pragma once

#include "common.cuh"
#include "kernel_tc.cuh"
#include "ptx.cuh"

namespace cgdr {

struct WyParams {
    const __nv_bfloat16* beta;  // [B, T, H]
    const float* g;             // [B, T, H] per-token log gate (nullptr: no gate)
    __nv_bfloat16* w;           // [B, T, H, K]
    __nv_bfloat16* u;           // [B, T, H, V]
    float* g_cum;               // [B, T, H] (nullptr: not stored)
    const int64_t* cu_seqlens;
    const int64_t* chunk_indices;
    int64_t B, T, H, HK, K, V, N, NT;
    int64_t nt_per_seq;
    int64_t n_tiles;
    int64_t b_sb, b_st, b_sh;   // beta strides
    int64_t g_sb, g_st, g_sh;
    int64_t c_sb, c_st, c_sh;   // g_cum strides
    int64_t w_sb, w_st, w_sh;
    int64_t u_sb, u_st, u_sh;
    int32_t varlen;
    int* status;
    uint64_t timeout_ns;
};

struct WyMaps {
    CUtensorMap k;  // dims (K, HK, T, B), box (64, 1, 64, 1)
    CUtensorMap v;  // dims (V, H, T, B),  box (64, 1, 64, 1)
};

struct WyArgs {
    WyMaps maps;
    WyParams p;
};

template <int K_, int V_, int STAGES>
struct WyConfig {
    static_assert(K_ == 64 || K_ == 128, "WY: K in {64, 128}");
    static_assert(V_ == 64 || V_ == 128, "WY: V in {64, 128}");
    static constexpr int kEpiWarps = 8;
    static constexpr int kEpiThreads = 32 * kEpiWarps;
    static constexpr int kThreads = 96 + kEpiThreads;
    static constexpr int kSubK = K_ / 64;
    static constexpr int kSubV = V_ / 64;
    static constexpr int kTileK = K_ * 128;   // [64 tokens][K] bf16
    static constexpr int kTileV = V_ * 128;   // [64 tokens][V] bf16
    static constexpr int kOffK = 0;           // within a stage
    static constexpr int kOffV = kTileK;
    static constexpr int kOffBeta = kTileK + kTileV;  // 64 fp32
    static constexpr int kOffGc = kOffBeta + 256;     // 64 fp32 (cumulative gate)
    static constexpr int kStageBytes = (kOffGc + 256 + 1023) / 1024 * 1024;
    static constexpr int kOffT = STAGES * kStageBytes;  // [2] bf16 T tiles [64][64], 128-byte swizzle
    static constexpr int kLd = 68;                       // fp32 row stride of A and Tf
    static constexpr int kOffA = kOffT + 2 * 8192;       // fp32 A [64][kLd]
    static constexpr int kOffTf = kOffA + 64 * kLd * 4;  // fp32 T [64][kLd]
    static constexpr int kOffY = kOffTf + 64 * kLd * 4;  // fp32 [3][16][16] block products
    static constexpr int kOffOutW = (kOffY + 3 * 256 * 4 + 1023) / 1024 * 1024;  // staging [64][K]
    static constexpr int kOffOutU = kOffOutW + kTileK;                            // staging [64][V]
    static constexpr int kOffBar = kOffOutU + kTileV;
    static constexpr int kNumBars = 2 * STAGES + 9;
    static constexpr int kUsed = kOffBar + kNumBars * 8 + 16;
    static constexpr int kSmemBytes = (kUsed + 1024 > 120 * 1024) ? kUsed + 1024 : 120 * 1024;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kAccStride = 256;
    static constexpr uint32_t kTmemU = 128;
    static constexpr uint32_t kTx = kTileK + kTileV;
    static constexpr uint32_t kIdescKK = umma_idesc_bf16(64, 64, false, false);
    static constexpr uint32_t kIdescW = umma_idesc_bf16(64, K_, false, true);
    static constexpr uint32_t kIdescU = umma_idesc_bf16(64, V_, false, true);
};

struct WyTile {
    int64_t b, t0, len, hv, kh;
    bool ok;
};

__device__ __forceinline__ WyTile wy_tile(const WyParams& p, int64_t tile)
{
    WyTile t;
    t.hv = tile % p.H;
    const int64_t row = tile / p.H;
    t.kh = t.hv / (p.H / p.HK);
    t.ok = true;
    if (p.varlen) {
        const int64_t n = p.chunk_indices[2 * row];
        const int64_t c = p.chunk_indices[2 * row + 1];
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
    } else {
        t.b = row / p.nt_per_seq;
        t.t0 = (row % p.nt_per_seq) * kChunk;
        t.len = p.T - t.t0 < kChunk ? p.T - t.t0 : kChunk;
    }
    return t;
}

__device__ __forceinline__ void wy_epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int K_, int V_, int STAGES>
__global__ void __launch_bounds__(352, 1) wy_tc_kernel(const __grid_constant__ WyArgs args)
{
    using Cfg = WyConfig<K_, V_, STAGES>;
    const WyParams& p = args.p;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;                 // [STAGES] k, v (TMA) + beta, g_c (gate loader)
    uint64_t* empty = bars + STAGES;       // [STAGES] W and U products done
    uint64_t* kk_full = bars + 2 * STAGES; // [2]
    uint64_t* t_ready = kk_full + 2;       // [2]
    uint64_t* wu_full = kk_full + 4;       // [2]
    uint64_t* acc_empty = kk_full + 6;     // [2]
    uint64_t* mma_drain = kk_full + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* never_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1 + 32);  // TMA bytes + the 32 gate-loader lanes
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&kk_full[a], 1);
            mbar_init(&t_ready[a], Cfg::kEpiWarps);
            mbar_init(&wu_full[a], 1);
            mbar_init(&acc_empty[a], Cfg::kEpiWarps);
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
        prefetch_tensormap(&args.maps.k);
        prefetch_tensormap(&args.maps.v);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const WaitCtl ctl{abort_flag, p.status, p.timeout_ns};
    const uint32_t sbase = smem_u32(smem);

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        int64_t it = 0;
        if (lane == 0) {
            for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
                const WyTile t = wy_tile(p, tile);
                if (!t.ok) {
                    if (p.status) atomicOr(p.status, 0x2);
                    continue;
                }
                const int s = static_cast<int>(it % STAGES);
                const uint32_t use = static_cast<uint32_t>(it / STAGES);
                if (it >= STAGES && !mbar_wait(&empty[s], (use - 1) & 1, ctl, 0x10)) break;
                uint8_t* st = smem + s * Cfg::kStageBytes;
                const int ib = static_cast<int>(t.b), it0 = static_cast<int>(t.t0);
                mbar_arrive_expect_tx(&full[s], Cfg::kTx);
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubK; ++sub)
                    tma_load_4d(&args.maps.k, st + Cfg::kOffK + sub * 8192, &full[s], sub * 64, static_cast<int>(t.kh),
                                it0, ib);
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubV; ++sub)
                    tma_load_4d(&args.maps.v, st + Cfg::kOffV + sub * 8192, &full[s], sub * 64, static_cast<int>(t.hv),
                                it0, ib);
                ++it;
            }
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            for (int64_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
                mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1, drain, 0x10);
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ gate loader
        int64_t it = 0;
        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const WyTile t = wy_tile(p, tile);
            if (!t.ok) continue;
            const int s = static_cast<int>(it % STAGES);
            const uint32_t use = static_cast<uint32_t>(it / STAGES);
            bool go = true;
            if (it >= STAGES && lane == 0) go = mbar_wait(&empty[s], (use - 1) & 1, ctl, 0x10);
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (!go) break;
            // rows 2*lane, 2*lane + 1; rows past the chunk's end read as beta = g = 0
            float be[2], gv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int r = 2 * lane + e;
                const int64_t tt = t.t0 + r;
                be[e] = r < t.len ? __bfloat162float(p.beta[t.b * p.b_sb + tt * p.b_st + t.hv * p.b_sh]) : 0.0f;
                gv[e] = (p.g && r < t.len) ? p.g[t.b * p.g_sb + tt * p.g_st + t.hv * p.g_sh] : 0.0f;
            }
            // inclusive scan in fp64, rounded once to fp32 (a CPU fp32 cumsum
            // accumulates in double: the reference's g_cum, benchmark.py:62)
            double x0 = gv[0], x1 = x0 + gv[1];
            double incl = x1;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, incl, d);
                if (lane >= d) incl += y;
            }
            double excl = __shfl_up_sync(0xffffffffu, incl, 1);
            if (lane == 0) excl = 0.0;
            const float c0 = static_cast<float>(excl + x0), c1 = static_cast<float>(incl);
            float* sb = reinterpret_cast<float*>(smem + s * Cfg::kStageBytes + Cfg::kOffBeta);
            float* sg = reinterpret_cast<float*>(smem + s * Cfg::kStageBytes + Cfg::kOffGc);
            sb[2 * lane] = be[0];
            sb[2 * lane + 1] = be[1];
            sg[2 * lane] = c0;
            sg[2 * lane + 1] = c1;
            if (p.g_cum) {
                if (2 * lane < t.len) p.g_cum[t.b * p.c_sb + (t.t0 + 2 * lane) * p.c_st + t.hv * p.c_sh] = c0;
                if (2 * lane + 1 < t.len) p.g_cum[t.b * p.c_sb + (t.t0 + 2 * lane + 1) * p.c_st + t.hv * p.c_sh] = c1;
            }
            mbar_arrive(&full[s]);
            ++it;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int64_t it = 0;
            for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
                const WyTile t = wy_tile(p, tile);
                if (!t.ok) continue;
                const int s = static_cast<int>(it % STAGES);
                const int a = static_cast<int>(it & 1);
                const uint32_t st = sbase + s * Cfg::kStageBytes;
                const uint32_t acc = tmem + a * Cfg::kAccStride;
                if (!mbar_wait(&full[s], static_cast<uint32_t>(it / STAGES) & 1, ctl, 0x20)) break;
                if (it >= 2 && !mbar_wait(&acc_empty[a], static_cast<uint32_t>(it / 2 - 1) & 1, ctl, 0x20)) break;
                tc_fence_after();
                {
                    const uint64_t d = umma_desc_sw128(st + Cfg::kOffK, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < K_ / 16; ++kk) {
                        const uint64_t off = static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
                        tc_mma_bf16(acc, d + off, d + off, Cfg::kIdescKK, kk > 0 ? 1u : 0u);
                    }
                }
                tc_commit(&kk_full[a]);
                if (!mbar_wait(&t_ready[a], static_cast<uint32_t>(it / 2) & 1, ctl, 0x20)) break;
                tc_fence_after();
                {
                    const uint64_t ta = umma_desc_sw128(sbase + Cfg::kOffT + a * 8192, 16, 1024);
                    const uint64_t kb = umma_desc_sw128(st + Cfg::kOffK, 8192, 1024);
                    const uint64_t vb = umma_desc_sw128(st + Cfg::kOffV, 8192, 1024);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_bf16(acc, ta + static_cast<uint64_t>((kk * 32) >> 4),
                                    kb + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescW, kk > 0 ? 1u : 0u);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_bf16(acc + Cfg::kTmemU, ta + static_cast<uint64_t>((kk * 32) >> 4),
                                    vb + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescU, kk > 0 ? 1u : 0u);
                }
                tc_commit(&wu_full[a]);
                tc_commit(&empty[s]);
                ++it;
            }
            tc_commit(mma_drain);
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            mbar_wait(mma_drain, 0, drain, 0x20);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int et = threadIdx.x - 96;     // 0..255
        const int ew = warp - 3;             // 0..7
        const int qd = warp & 3;             // TMEM lane quadrant
        const int ch = ew >> 2;              // column half
        const int ra = 16 * qd + (lane >> 2);
        const int rb = ra + 8;
        const int pc = 2 * (lane & 3);
        float* Am = reinterpret_cast<float*>(smem + Cfg::kOffA);
        float* Tf = reinterpret_cast<float*>(smem + Cfg::kOffTf);
        float* Yb = reinterpret_cast<float*>(smem + Cfg::kOffY);
        constexpr int LD = Cfg::kLd;
        bool ok = true;
        int64_t it = 0;
        WyTile prev{};

        // w, u of the tile with index j (accumulator set j % 2)
        auto output = [&](int64_t j, const WyTile& t) {
            const int a = static_cast<int>(j & 1);
            const uint32_t acc = tmem + a * Cfg::kAccStride + ((32u * qd) << 16);
            if (ok) ok = mbar_wait(&wu_full[a], static_cast<uint32_t>(j / 2) & 1, ctl, 0x40);
            ok = __all_sync(0xffffffffu, ok) != 0;
            constexpr int kWc = K_ / 2, kUc = V_ / 2;  // columns of W / U per warp
            uint32_t rw[kWc / 32][16], ru[kUc / 32][16];
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int cb = 0; cb < kWc / 32; ++cb)
                    tmem_ld_16x256b_x4(acc + static_cast<uint32_t>(kWc * ch + 32 * cb), rw[cb]);
#pragma unroll
                for (int cb = 0; cb < kUc / 32; ++cb)
                    tmem_ld_16x256b_x4(acc + Cfg::kTmemU + static_cast<uint32_t>(kUc * ch + 32 * cb), ru[cb]);
                tmem_wait_ld();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
            wy_epi_bar();  // staging free: every thread stored the previous tile's rows
            uint8_t* sw = smem + Cfg::kOffOutW;
            uint8_t* su = smem + Cfg::kOffOutU;
            if (ok) {
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int i = half ? rb : ra;
#pragma unroll
                        for (int cb = 0; cb < kWc / 32; ++cb)
                            *reinterpret_cast<uint32_t*>(sw + sw128_off(i, kWc * ch + 32 * cb + 8 * jj + pc, 8192)) =
                                pack_bf16x2(__uint_as_float(rw[cb][4 * jj + 2 * half]),
                                            __uint_as_float(rw[cb][4 * jj + 2 * half + 1]));
#pragma unroll
                        for (int cb = 0; cb < kUc / 32; ++cb)
                            *reinterpret_cast<uint32_t*>(su + sw128_off(i, kUc * ch + 32 * cb + 8 * jj + pc, 8192)) =
                                pack_bf16x2(__uint_as_float(ru[cb][4 * jj + 2 * half]),
                                            __uint_as_float(ru[cb][4 * jj + 2 * half + 1]));
                    }
            }
            wy_epi_bar();
            if (ok) {
                __nv_bfloat16* wr = p.w + t.b * p.w_sb + t.t0 * p.w_st + t.hv * p.w_sh;
                __nv_bfloat16* ur = p.u + t.b * p.u_sb + t.t0 * p.u_st + t.hv * p.u_sh;
#pragma unroll
                for (int e = et; e < 64 * (K_ / 8); e += Cfg::kEpiThreads) {
                    const int row = e / (K_ / 8), cc = e % (K_ / 8);
                    if (row < t.len)
                        *reinterpret_cast<uint4*>(wr + row * p.w_st + 8 * cc) =
                            *reinterpret_cast<const uint4*>(sw + sw128_off(row, 8 * cc, 8192));
                }
#pragma unroll
                for (int e = et; e < 64 * (V_ / 8); e += Cfg::kEpiThreads) {
                    const int row = e / (V_ / 8), cc = e % (V_ / 8);
                    if (row < t.len)
                        *reinterpret_cast<uint4*>(ur + row * p.u_st + 8 * cc) =
                            *reinterpret_cast<const uint4*>(su + sw128_off(row, 8 * cc, 8192));
                }
            }
        };

        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const WyTile t = wy_tile(p, tile);
            if (!t.ok) continue;
            const int s = static_cast<int>(it % STAGES);
            const int a = static_cast<int>(it & 1);
            uint8_t* st = smem + s * Cfg::kStageBytes;
            const float* sb = reinterpret_cast<const float*>(st + Cfg::kOffBeta);
            const float* sg = reinterpret_cast<const float*>(st + Cfg::kOffGc);
            if (ok) ok = mbar_wait(&full[s], static_cast<uint32_t>(it / STAGES) & 1, ctl, 0x40);
            if (ok) ok = mbar_wait(&kk_full[a], static_cast<uint32_t>(it / 2) & 1, ctl, 0x40);
            ok = __all_sync(0xffffffffu, ok) != 0;
            // ---- A = bf16(k k^T) * beta_i * exp(g_i - g_j), strictly lower, rows/cols < len
            if (ok) {
                tc_fence_after();
                uint32_t kr[16];
                tmem_ld_16x256b_x4(tmem + a * Cfg::kAccStride + ((32u * qd) << 16) + 32 * ch, kr);
                // k' = bf16(beta * exp(g_c) * k), v' = bf16(beta * v) in place (rows past the
                // chunk's end become 0); thread et handles row et/4, a quarter of each row
                {
                    const int r = et >> 2, qt = et & 3;
                    const bool live = r < t.len;
                    const float br = sb[r];
                    const float fk = live ? __fmul_rn(br, expf(sg[r])) : 0.0f;
                    constexpr int kCk = K_ / 32, kCv = V_ / 32;  // 16-byte chunks per quarter row
#pragma unroll
                    for (int c = 0; c < kCk; ++c) {
                        const int idx = qt * kCk + ((c + r) & (kCk - 1));
                        uint8_t* ptr = st + Cfg::kOffK + (idx >> 3) * 8192 + r * 128 + (idx & 7) * 16;
                        uint4 x = *reinterpret_cast<const uint4*>(ptr);
                        uint32_t* xs = &x.x;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 v = unpack_bf16x2(xs[e]);
                            xs[e] = live ? pack_bf16x2(__fmul_rn(fk, v.x), __fmul_rn(fk, v.y)) : 0u;
                        }
                        *reinterpret_cast<uint4*>(ptr) = x;
                    }
#pragma unroll
                    for (int c = 0; c < kCv; ++c) {
                        const int idx = qt * kCv + ((c + r) & (kCv - 1));
                        uint8_t* ptr = st + Cfg::kOffV + (idx >> 3) * 8192 + r * 128 + (idx & 7) * 16;
                        uint4 x = *reinterpret_cast<const uint4*>(ptr);
                        uint32_t* xs = &x.x;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 v = unpack_bf16x2(xs[e]);
                            xs[e] = live ? pack_bf16x2(__fmul_rn(v.x, br), __fmul_rn(v.y, br)) : 0u;
                        }
                        *reinterpret_cast<uint4*>(ptr) = x;
                    }
                }
                tmem_wait_ld();
                const float ba = sb[ra], bb = sb[rb], ga = sg[ra], gb = sg[rb];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int i = half ? rb : ra;
                        const float bi = half ? bb : ba, gi = half ? gb : ga;
#pragma unroll
                        for (int bit = 0; bit < 2; ++bit) {
                            const int j = 32 * ch + 8 * jj + pc + bit;
                            const float kk = round_bf16(__uint_as_float(kr[4 * jj + 2 * half + bit]));
                            float x = 0.0f;
                            if (j < i && i < t.len) x = __fmul_rn(__fmul_rn(kk, bi), expf(gi - sg[j]));
                            Am[i * LD + j] = x;
                        }
                    }
            }
            wy_epi_bar();
            // ---- T = (I + A)^-1: the four 16 x 16 diagonal blocks, one warp each,
            // lane c < 16 owning column c of its block (forward substitution)
            if (ok && ew < 4) {
                const int b0 = 16 * ew, c = lane & 15;
                float tcol[16];
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    float acc = 0.0f;
#pragma unroll
                    for (int m = 0; m < r; ++m) acc = fmaf(Am[(b0 + r) * LD + b0 + m], tcol[m], acc);
                    tcol[r] = (r == c) ? 1.0f : -acc;
                }
                if (lane < 16) {
#pragma unroll
                    for (int r = 0; r < 16; ++r) Tf[(b0 + r) * LD + b0 + c] = (r < c) ? 0.0f : tcol[r];
                }
            }
            wy_epi_bar();
            // ---- blocks below the diagonal, one diagonal d at a time:
            //      Y_ij = sum_{m=j}^{i-1} A_im T_mj ;  T_ij = -T_ii Y_ij
            for (int d = 1; d < 4; ++d) {
                const int nb = 4 - d;  // blocks on this diagonal: (j + d, j), j = 0 .. nb-1
                const int r = et >> 4, c = et & 15;
                if (ok) {
                    for (int bj = 0; bj < nb; ++bj) {
                        const int bi = bj + d;
                        float acc = 0.0f;
                        for (int bm = bj; bm < bi; ++bm)
#pragma unroll
                            for (int k = 0; k < 16; ++k)
                                acc = fmaf(Am[(16 * bi + r) * LD + 16 * bm + k], Tf[(16 * bm + k) * LD + 16 * bj + c], acc);
                        Yb[bj * 256 + r * 16 + c] = acc;
                    }
                }
                wy_epi_bar();
                if (ok) {
                    for (int bj = 0; bj < nb; ++bj) {
                        const int bi = bj + d;
                        float acc = 0.0f;
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            acc = fmaf(Tf[(16 * bi + r) * LD + 16 * bi + k], Yb[bj * 256 + k * 16 + c], acc);
                        Tf[(16 * bi + r) * LD + 16 * bj + c] = -acc;
                    }
                }
                wy_epi_bar();
            }
            // ---- T -> bf16 tile (128-byte swizzle, K-major A operand of the W / U products)
            if (ok) {
                uint8_t* tt = smem + Cfg::kOffT + a * 8192;
                const int r = et >> 2, c0 = 16 * (et & 3);
#pragma unroll
                for (int c = 0; c < 16; c += 8) {
                    uint4 v;
                    const float* src = Tf + r * LD + c0 + c;
                    v.x = pack_bf16x2(c0 + c + 0 <= r ? src[0] : 0.0f, c0 + c + 1 <= r ? src[1] : 0.0f);
                    v.y = pack_bf16x2(c0 + c + 2 <= r ? src[2] : 0.0f, c0 + c + 3 <= r ? src[3] : 0.0f);
                    v.z = pack_bf16x2(c0 + c + 4 <= r ? src[4] : 0.0f, c0 + c + 5 <= r ? src[5] : 0.0f);
                    v.w = pack_bf16x2(c0 + c + 6 <= r ? src[6] : 0.0f, c0 + c + 7 <= r ? src[7] : 0.0f);
                    *reinterpret_cast<uint4*>(tt + sw128_off(r, c0 + c, 8192)) = v;
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_ready[a]);
            // ---- the previous tile's w and u
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
