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
// of a unit lower-triangular matrix, in fp32: forward substitution inside the
// four 16 x 16 diagonal blocks T_ii, then with B_im = T_ii A_im block forward
// substitution T_ij = -sum_{m=j}^{i-1} B_im T_mj, where the three-deep block
// T_30 is folded into two steps, T_30 = -(C_30 T_00 + C_31 T_10) with
// C_3m = B_3m - B_32 B_2m (substituting T_20).
//
// The reference rounds k' = beta * exp(g_c) * k and v' = beta * v to bf16 and
// multiplies them by bf16(T).  Here the row factors move onto T's columns:
// W = bf16(T diag(beta e^g_c)) . k and U = bf16(T diag(beta)) . v, so k and v
// go to the tensor cores as TMA delivered them; the two orders differ at the
// bf16 rounding of the operands.
//
// Persistent kernel, one CTA per SM walking tiles (chunk row, value head)
// blockIdx.x, blockIdx.x + gridDim.x, ...  Warp roles (608 threads):
//   warp 0      TMA producer: k and v of a tile into a STAGES-deep ring;
//   warp 1      TMEM owner (512 columns: two sets of W [64 x K] at +0 and
//               U [64 x V] at +128, 256 apart; k k^T is written into W's first
//               64 columns and read before W's product overwrites it);
//   warp 2      gate loader: beta and g of the tile (plain loads), the fp64
//               cumulative sum, the g_c output, both into the stage;
//   warps 3-18  two epilogue groups of eight warps (two per TMEM lane quadrant:
//               warp w reads lanes 32(w%4).., rows 16(w%4)..+15 of an M=64
//               accumulator, and half of the columns).  Group g takes the tiles
//               of accumulator set g (every other tile), so two tiles are solved
//               at once, each group with its own scratch and named barrier.
//               The group's first warp issues that group's MMAs (one elected
//               lane), so a group never waits on the other group's progress.
// Per tile (stage s, accumulator set a = group):
//   MMA   KK[a] = k k^T                       M=64 N=64 K=K (both K-major)
//   epi   A; T (diagonal 16 x 16 blocks one per warp, then the blocks below the
//         diagonal); T' = bf16(T diag(beta e^g_c)), T'' = bf16(T diag(beta))
//   MMA   W[a] = T' k ; U[a] = T'' v          M=64 N=K / V K=64 (B MN-major)
//   epi   w, u = bf16 from TMEM (16x256b loads, quad transpose) -> 16-byte stores
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
    static constexpr int kEpiWarps = 16;  // two groups of eight
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
    static constexpr int kOffD = kOffGc + 256;        // 64 fp32: beta * exp(g_c), T' column factors
    static constexpr int kOffInfo = kOffD + 256;      // WyStageInfo of the tile in this stage
    static constexpr int kStageBytes = (kOffInfo + 32 + 1023) / 1024 * 1024;
    static constexpr int kOffT = STAGES * kStageBytes;  // [2 sets][T', T''] bf16 [64][64], 128-byte swizzle
    static constexpr int kLd = 68;                       // fp32 row stride of A and Tf
    static constexpr int kLdY = 20;                      // row stride of a B block: 8 rows hit 8 banks
    static constexpr int kScratch = 2 * 64 * kLd * 4 + 7 * 16 * kLdY * 4;  // A, Tf, Y [7][16][kLdY] of a group
    static constexpr int kOffScratch = kOffT + 4 * 8192;             // [2 groups]
    static constexpr int kOffBar = (kOffScratch + 2 * kScratch + 1023) / 1024 * 1024;
    static constexpr int kNumBars = 2 * STAGES + 6;
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

// The tile a stage holds, decoded once by the gate loader; `end` marks the
// two slots after a CTA's last tile (one per epilogue group).
struct WyStageInfo {
    int32_t b, t0, len, hv, end;
};

struct WyTile {
    int64_t b, t0, len, hv, kh;
    bool ok;
    bool pad;  // chunk_indices row (-1, -1): a padding row, skipped without a flag
};

__device__ __forceinline__ WyTile wy_tile(const WyParams& p, int64_t tile)
{
    WyTile t;
    t.hv = tile % p.H;
    const int64_t row = tile / p.H;
    t.kh = t.hv / (p.H / p.HK);
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
    } else {
        t.b = row / p.nt_per_seq;
        t.t0 = (row % p.nt_per_seq) * kChunk;
        t.len = p.T - t.t0 < kChunk ? p.T - t.t0 : kChunk;
    }
    return t;
}

// 4 x 4 transpose of 32-bit values across the lanes of a quad: lane i's a[j]
// becomes lane j's a[i] (two butterfly rounds, four shuffles).
__device__ __forceinline__ void quad_transpose(uint32_t (&a)[4], int lane)
{
    const bool o1 = lane & 1, o2 = lane & 2;
    uint32_t r0 = __shfl_xor_sync(0xffffffffu, o1 ? a[0] : a[1], 1);
    uint32_t r1 = __shfl_xor_sync(0xffffffffu, o1 ? a[2] : a[3], 1);
    if (o1) {
        a[0] = r0;
        a[2] = r1;
    } else {
        a[1] = r0;
        a[3] = r1;
    }
    r0 = __shfl_xor_sync(0xffffffffu, o2 ? a[0] : a[2], 2);
    r1 = __shfl_xor_sync(0xffffffffu, o2 ? a[1] : a[3], 2);
    if (o2) {
        a[0] = r0;
        a[1] = r1;
    } else {
        a[2] = r0;
        a[3] = r1;
    }
}

// named barrier of epilogue group g (ids 1 and 2, 256 threads each)
__device__ __forceinline__ void wy_group_bar(int g) { asm volatile("bar.sync %0, 256;" ::"r"(1 + g) : "memory"); }

__device__ __forceinline__ void fma4(float4& y, float a, const float4& b)
{
    y.x = fmaf(a, b.x, y.x);
    y.y = fmaf(a, b.y, y.y);
    y.z = fmaf(a, b.z, y.z);
    y.w = fmaf(a, b.w, y.w);
}

// 16 x 16 block products in fp32 from shared memory (L, R: the blocks' first
// elements, row strides in floats; 16-byte aligned rows).
// y[h] += (L R)[r + 8h][c4..c4+3]
__device__ __forceinline__ void wy_prod24(const float* L, int ldl, const float* R, int ldr, int r, int c4,
                                          float4 (&y)[2])
{
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
        const float4 l0 = *reinterpret_cast<const float4*>(L + r * ldl + 4 * k4);
        const float4 l1 = *reinterpret_cast<const float4*>(L + (r + 8) * ldl + 4 * k4);
        const float a0[4] = {l0.x, l0.y, l0.z, l0.w}, a1[4] = {l1.x, l1.y, l1.z, l1.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float4 b = *reinterpret_cast<const float4*>(R + (4 * k4 + e) * ldr + c4);
            fma4(y[0], a0[e], b);
            fma4(y[1], a1[e], b);
        }
    }
}
// y += (L R)[r][c4..c4+3]
__device__ __forceinline__ void wy_prod14(const float* L, int ldl, const float* R, int ldr, int r, int c4, float4& y)
{
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
        const float4 l = *reinterpret_cast<const float4*>(L + r * ldl + 4 * k4);
        const float a[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) fma4(y, a[e], *reinterpret_cast<const float4*>(R + (4 * k4 + e) * ldr + c4));
    }
}

// the same barrier, returning whether `v` holds in every thread of the group
__device__ __forceinline__ bool wy_group_bar_and(int g, bool v)
{
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n"
        " setp.ne.u32 q, %1, 0;\n"
        " bar.red.and.pred p, %2, 256, q;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"(v ? 1u : 0u), "r"(1 + g)
        : "memory");
    return r != 0;
}

template <int K_, int V_, int STAGES>
__global__ void __launch_bounds__(608, 1) wy_tc_kernel(const __grid_constant__ WyArgs args)
{
    using Cfg = WyConfig<K_, V_, STAGES>;
    const WyParams& p = args.p;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;                 // [STAGES] k, v (TMA) + beta, g_c (gate loader)
    uint64_t* empty = bars + STAGES;       // [STAGES] W and U products done
    uint64_t* kk_full = bars + 2 * STAGES; // [2]
    uint64_t* wu_full = kk_full + 2;       // [2]
    uint64_t* mma_drain = kk_full + 4;     // [2]
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
            mbar_init(&wu_full[a], 1);
            mbar_init(&mma_drain[a], 1);
        }
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
                    if (p.status && !t.pad) atomicOr(p.status, 0x2);
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
            // the two end slots carry no bytes
            for (int e = 0; e < 2 && !*abort_flag; ++e, ++it) {
                const int s = static_cast<int>(it % STAGES);
                if (it >= STAGES && !mbar_wait(&empty[s], (static_cast<uint32_t>(it / STAGES) - 1) & 1, ctl, 0x10)) break;
                mbar_arrive(&full[s]);
            }
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            for (int64_t j = it > STAGES ? it - STAGES : 0; j < it; ++j)
                mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1, drain, 0x10);
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ gate loader
        int64_t it = 0;
        bool alive = true;
        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const WyTile t = wy_tile(p, tile);
            if (!t.ok) continue;
            const int s = static_cast<int>(it % STAGES);
            const uint32_t use = static_cast<uint32_t>(it / STAGES);
            bool go = true;
            if (it >= STAGES && lane == 0) go = mbar_wait(&empty[s], (use - 1) & 1, ctl, 0x10);
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (!go) {
                alive = false;
                break;
            }
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
            float* sd = reinterpret_cast<float*>(smem + s * Cfg::kStageBytes + Cfg::kOffD);
            if (lane == 0)
                *reinterpret_cast<WyStageInfo*>(smem + s * Cfg::kStageBytes + Cfg::kOffInfo) =
                    WyStageInfo{static_cast<int32_t>(t.b), static_cast<int32_t>(t.t0), static_cast<int32_t>(t.len),
                                static_cast<int32_t>(t.hv), 0};
            sb[2 * lane] = be[0];
            sb[2 * lane + 1] = be[1];
            sg[2 * lane] = c0;
            sg[2 * lane + 1] = c1;
            sd[2 * lane] = __fmul_rn(be[0], expf(c0));
            sd[2 * lane + 1] = __fmul_rn(be[1], expf(c1));
            if (p.g_cum) {
                if (2 * lane < t.len) p.g_cum[t.b * p.c_sb + (t.t0 + 2 * lane) * p.c_st + t.hv * p.c_sh] = c0;
                if (2 * lane + 1 < t.len) p.g_cum[t.b * p.c_sb + (t.t0 + 2 * lane + 1) * p.c_st + t.hv * p.c_sh] = c1;
            }
            mbar_arrive(&full[s]);
            ++it;
        }
        for (int e = 0; e < 2 && alive; ++e, ++it) {
            const int s = static_cast<int>(it % STAGES);
            bool go = *abort_flag == 0;
            if (go && it >= STAGES && lane == 0)
                go = mbar_wait(&empty[s], (static_cast<uint32_t>(it / STAGES) - 1) & 1, ctl, 0x10);
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (!go) break;
            if (lane == 0) reinterpret_cast<WyStageInfo*>(smem + s * Cfg::kStageBytes + Cfg::kOffInfo)->end = 1;
            mbar_arrive(&full[s]);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ TMEM owner
        // (allocated above, released at the end; the groups issue their own MMAs)
    } else {
        // ------------------------------------------------------------ epilogue
        const int grp = (warp - 3) >> 3;     // group: accumulator set, every other tile
        const int gw = (warp - 3) & 7;       // warp within the group
        const int gt = 32 * gw + lane;       // thread within the group, 0..255
        const int qd = warp & 3;             // TMEM lane quadrant
        const int ch = gw >> 2;              // column half (two warps per quadrant)
        const int ra = 16 * qd + (lane >> 2);
        const int rb = ra + 8;
        const int pc = 2 * (lane & 3);
        uint8_t* scratch = smem + Cfg::kOffScratch + grp * Cfg::kScratch;
        float* Am = reinterpret_cast<float*>(scratch);
        float* Tf = Am + 64 * Cfg::kLd;
        float* Yb = Tf + 64 * Cfg::kLd;
        constexpr int LD = Cfg::kLd;
        const uint32_t acc = tmem + grp * Cfg::kAccStride;
        // the group's first warp issues its MMAs and commits: the whole warp runs that
        // code (warp-uniform descriptors) and one elected lane issues
        const bool issuer = gw == 0;
        const uint32_t tw_addr = sbase + Cfg::kOffT + (2 * grp) * 8192;
        bool ok = true;
        // slot `my` of the stage ring (this CTA's valid tiles in order, then two end
        // slots); this group takes the slots my % 2 == grp
        for (int64_t my = grp;; my += 2) {
            const int s = static_cast<int>(my % STAGES);
            const uint32_t par = static_cast<uint32_t>(my / 2) & 1;
            uint8_t* st = smem + s * Cfg::kStageBytes;
            const float* sb = reinterpret_cast<const float*>(st + Cfg::kOffBeta);
            const float* sg = reinterpret_cast<const float*>(st + Cfg::kOffGc);
            const float* sd = reinterpret_cast<const float*>(st + Cfg::kOffD);
            if (ok) ok = mbar_wait(&full[s], static_cast<uint32_t>(my / STAGES) & 1, ctl, 0x40);
            // the whole group agrees to go on (and has finished reading the previous
            // tile's accumulators, so KK may overwrite them)
            tc_fence_before();
            if (!wy_group_bar_and(grp, ok)) break;
            const WyStageInfo info = *reinterpret_cast<const WyStageInfo*>(st + Cfg::kOffInfo);
            if (info.end) break;
            WyTile t;
            t.b = info.b;
            t.t0 = info.t0;
            t.len = info.len;
            t.hv = info.hv;
            // KK = k k^T into W's first 64 columns
            if (issuer) {
                tc_fence_after();
                const uint64_t d = umma_desc_sw128(sbase + s * Cfg::kStageBytes + Cfg::kOffK, 16, 1024);
                if (elect_one_sync()) {
#pragma unroll
                    for (int kk = 0; kk < K_ / 16; ++kk) {
                        const uint64_t off = static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
                        tc_mma_bf16(acc, d + off, d + off, Cfg::kIdescKK, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&kk_full[grp]);
                }
                __syncwarp();
            }
            if (ok) ok = mbar_wait(&kk_full[grp], par, ctl, 0x40);
            ok = __all_sync(0xffffffffu, ok) != 0;
            // ---- A = bf16(k k^T) * beta_i * exp(g_i - g_j), strictly lower, rows < len
            if (ok) {
                tc_fence_after();
                uint32_t kr[16];
                tmem_ld_16x256b_x4(acc + ((32u * qd) << 16) + 32 * ch, kr);
                const float ba = sb[ra], bb = sb[rb], ga = sg[ra], gb = sg[rb];
                tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                        for (int half = 0; half < 2; ++half) {
                            const int i = half ? rb : ra;
                            const float bi = half ? bb : ba, gi = half ? gb : ga;
                            const int j = 32 * ch + 8 * jj + pc;
                            float x[2];
#pragma unroll
                            for (int bit = 0; bit < 2; ++bit) {
                                const float kk = round_bf16(__uint_as_float(kr[4 * jj + 2 * half + bit]));
                                x[bit] = (j + bit < i && i < t.len)
                                             ? __fmul_rn(__fmul_rn(kk, bi), __expf(gi - sg[j + bit]))
                                             : 0.0f;
                            }
                            *reinterpret_cast<float2*>(Am + i * LD + j) = make_float2(x[0], x[1]);
                        }
            }
            tc_fence_before();
            wy_group_bar(grp);
            // ---- T = (I + A)^-1, diagonal blocks: warp gw < 4 owns block gw, lane c (and
            // c + 16) column c; forward substitution row by row,
            // T[m][c] = -sum_{l<m} A[m][l] T[l][c] accumulated in increasing l (row m of
            // A read as broadcast 16-byte loads)
            if (ok && gw < 4) {
                const int b0 = 16 * gw, c = lane & 15;
                float x[16];
#pragma unroll
                for (int m = 0; m < 16; ++m) {
                    const float4* arow = reinterpret_cast<const float4*>(Am + (b0 + m) * LD + b0);
                    float acc = 0.0f;
#pragma unroll
                    for (int q = 0; q < (m + 3) / 4; ++q) {
                        const float4 a4 = arow[q];
                        if (4 * q + 0 < m) acc = fmaf(a4.x, x[4 * q + 0], acc);
                        if (4 * q + 1 < m) acc = fmaf(a4.y, x[4 * q + 1], acc);
                        if (4 * q + 2 < m) acc = fmaf(a4.z, x[4 * q + 2], acc);
                        if (4 * q + 3 < m) acc = fmaf(a4.w, x[4 * q + 3], acc);
                    }
                    x[m] = (m == c) ? 1.0f : (m < c ? 0.0f : -acc);
                }
                if (lane < 16) {
#pragma unroll
                    for (int r = 0; r < 16; ++r) Tf[(b0 + r) * LD + b0 + c] = x[r];
                }
            }
            wy_group_bar(grp);
            // ---- blocks below the diagonal: B_im = T_ii A_im for the six pairs m < i,
            // then per diagonal d: T_ij = -sum_{m=j}^{i-1} B_im T_mj
            // (one warp per pair, thread rows r8 and r8 + 8, columns c4..c4+3)
            const int r = (gt >> 2) & 15, c4 = 4 * (gt & 3), sub = gt >> 6;  // the steps' thread layout
            if (ok && gw < 6) {
                const int pidx = gw;  // pairs (1,0) (2,0) (2,1) (3,0) (3,1) (3,2)
                const int bi = pidx == 0 ? 1 : (pidx < 3 ? 2 : 3);
                const int bm = pidx == 0 ? 0 : (pidx < 3 ? pidx - 1 : pidx - 3);
                const int r8 = lane >> 2, c4q = 4 * (lane & 3);
                float4 y[2] = {};
                wy_prod24(Tf + 16 * bi * LD + 16 * bi, LD, Am + 16 * bi * LD + 16 * bm, LD, r8, c4q, y);
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    *reinterpret_cast<float4*>(Yb + pidx * 16 * Cfg::kLdY + (r8 + 8 * h) * Cfg::kLdY + c4q) = y[h];
            }
            wy_group_bar(grp);
            // ---- block forward substitution T_ij = -sum_{m=j}^{i-1} B_im T_mj in two
            // steps: the third diagonal is folded into the second by substituting T_20,
            // T_30 = -(C_30 T_00 + C_31 T_10) with C_3m = B_3m - B_32 B_2m.
            // B slots: 0 B_10, 1 B_20, 2 B_21, 3 B_30 (then C_30), 4 B_31, 5 B_32, 6 C_31.
            auto yslot = [&](int k) { return Yb + k * 16 * Cfg::kLdY; };
            auto tblk = [&](int bi, int bj) { return Tf + 16 * bi * LD + 16 * bj; };
            // step 1: T_10, T_21, T_32 (two warps each, thread row r, columns c4..c4+3);
            // C_30, C_31 (one warp each, rows r8 and r8 + 8)
            if (ok) {
                if (sub < 3) {
                    const int bj = sub;  // T_{bj+1, bj} = -B_{bj+1, bj} T_{bj, bj}
                    float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    wy_prod14(yslot(bj == 0 ? 0 : bj == 1 ? 2 : 5), Cfg::kLdY, tblk(bj, bj), LD, r, c4, y);
                    *reinterpret_cast<float4*>(tblk(bj + 1, bj) + r * LD + c4) = make_float4(-y.x, -y.y, -y.z, -y.w);
                } else {
                    const int m = gw - 6, r8 = lane >> 2, c4q = 4 * (lane & 3);  // C_3m = B_3m - B_32 B_2m
                    float4 y[2] = {};
                    wy_prod24(yslot(5), Cfg::kLdY, yslot(1 + m), Cfg::kLdY, r8, c4q, y);
                    const float* bsrc = yslot(3 + m);
                    float* dst = yslot(m == 0 ? 3 : 6);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int row = r8 + 8 * h;
                        const float4 b = *reinterpret_cast<const float4*>(bsrc + row * Cfg::kLdY + c4q);
                        *reinterpret_cast<float4*>(dst + row * Cfg::kLdY + c4q) =
                            make_float4(b.x - y[h].x, b.y - y[h].y, b.z - y[h].z, b.w - y[h].w);
                    }
                }
            }
            wy_group_bar(grp);
            // step 2: T_20 = -(B_20 T_00 + B_21 T_10), T_31 = -(B_31 T_11 + B_32 T_21),
            // T_30 = -(C_30 T_00 + C_31 T_10) (two warps each)
            if (ok && sub < 3) {
                const float* L1 = yslot(sub == 0 ? 1 : sub == 1 ? 4 : 3);
                const float* L2 = yslot(sub == 0 ? 2 : sub == 1 ? 5 : 6);
                const float* R1 = sub == 1 ? tblk(1, 1) : tblk(0, 0);
                const float* R2 = sub == 1 ? tblk(2, 1) : tblk(1, 0);
                float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                wy_prod14(L1, Cfg::kLdY, R1, LD, r, c4, y);
                wy_prod14(L2, Cfg::kLdY, R2, LD, r, c4, y);
                float* D = sub == 0 ? tblk(2, 0) : sub == 1 ? tblk(3, 1) : tblk(3, 0);
                *reinterpret_cast<float4*>(D + r * LD + c4) = make_float4(-y.x, -y.y, -y.z, -y.w);
            }
            wy_group_bar(grp);
            // ---- T' = bf16(T diag(beta e^g_c)), T'' = bf16(T diag(beta)) (128-byte
            // swizzle, K-major A operands); thread: row gt/4, 16 columns
            if (ok) {
                uint8_t* tw = smem + Cfg::kOffT + (2 * grp) * 8192;
                uint8_t* tu = tw + 8192;
                const int row = gt >> 2, cb0 = 16 * (gt & 3);
                const float4* t4p = reinterpret_cast<const float4*>(Tf + row * LD + cb0);
                const float4* b4p = reinterpret_cast<const float4*>(sb + cb0);
                const float4* d4p = reinterpret_cast<const float4*>(sd + cb0);
#pragma unroll
                for (int cg8 = 0; cg8 < 2; ++cg8) {
                    const int c0 = cb0 + 8 * cg8;
                    uint32_t pw[4], pu[4];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int c = c0 + 4 * h;  // T is lower triangular: columns past the row are 0
                        const float4 t4 = t4p[2 * cg8 + h], b4 = b4p[2 * cg8 + h], d4 = d4p[2 * cg8 + h];
                        const float t0 = c <= row ? t4.x : 0.0f, t1 = c + 1 <= row ? t4.y : 0.0f;
                        const float t2 = c + 2 <= row ? t4.z : 0.0f, t3 = c + 3 <= row ? t4.w : 0.0f;
                        pw[2 * h] = pack_bf16x2(__fmul_rn(t0, d4.x), __fmul_rn(t1, d4.y));
                        pw[2 * h + 1] = pack_bf16x2(__fmul_rn(t2, d4.z), __fmul_rn(t3, d4.w));
                        pu[2 * h] = pack_bf16x2(__fmul_rn(t0, b4.x), __fmul_rn(t1, b4.y));
                        pu[2 * h + 1] = pack_bf16x2(__fmul_rn(t2, b4.z), __fmul_rn(t3, b4.w));
                    }
                    *reinterpret_cast<uint4*>(tw + sw128_off(row, c0, 8192)) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
                    *reinterpret_cast<uint4*>(tu + sw128_off(row, c0, 8192)) = make_uint4(pu[0], pu[1], pu[2], pu[3]);
                }
                if (t.len < kChunk) {
                    // rows of k and v past the chunk's end belong to another sequence (or
                    // are fill): zero them so that no value of theirs reaches a product
                    const int rows = kChunk - static_cast<int>(t.len);
                    for (int e = gt; e < (Cfg::kSubK + Cfg::kSubV) * rows * 8; e += 256) {
                        const int tsub = e / (rows * 8), rr = static_cast<int>(t.len) + (e / 8) % rows, c8 = e & 7;
                        uint8_t* base = tsub < Cfg::kSubK ? st + Cfg::kOffK + tsub * 8192
                                                          : st + Cfg::kOffV + (tsub - Cfg::kSubK) * 8192;
                        *reinterpret_cast<uint4*>(base + rr * 128 + c8 * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            wy_group_bar(grp);
            // W = T' k, U = T'' v (M=64, N=K / V, K=64; k and v MN-major); the stage
            // is free once they complete
            if (issuer && ok) {
                tc_fence_after();
                const uint32_t st = sbase + s * Cfg::kStageBytes;
                const uint64_t tw = umma_desc_sw128(tw_addr, 16, 1024);
                const uint64_t tu = umma_desc_sw128(tw_addr + 8192, 16, 1024);
                const uint64_t kb = umma_desc_sw128(st + Cfg::kOffK, 8192, 1024);
                const uint64_t vb = umma_desc_sw128(st + Cfg::kOffV, 8192, 1024);
                if (elect_one_sync()) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_bf16(acc, tw + static_cast<uint64_t>((kk * 32) >> 4),
                                    kb + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescW, kk > 0 ? 1u : 0u);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_bf16(acc + Cfg::kTmemU, tu + static_cast<uint64_t>((kk * 32) >> 4),
                                    vb + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdescU, kk > 0 ? 1u : 0u);
                    tc_commit(&wu_full[grp]);
                    tc_commit(&empty[s]);
                }
                __syncwarp();
            }
            // ---- w, u: 16x256b fragments (thread: rows ra, rb; column pairs 2(lane%4) of
            // each 8-column group) in two batches (w, then u), a quad transpose turns the
            // pairs into 16-byte chunks (lane l%4 takes the group l%4 of every 32 columns)
            if (ok) ok = mbar_wait(&wu_full[grp], par, ctl, 0x40);
            ok = __all_sync(0xffffffffu, ok) != 0;
            if (ok) {
                tc_fence_after();
                const int qi = lane & 3;
                const bool live_a = ra < t.len, live_b = rb < t.len;
#pragma unroll
                for (int batch = 0; batch < 2; ++batch) {
                    constexpr int kMaxBlk = 2;                 // this warp: half of the columns
                    const int ncols = (batch == 0 ? K_ : V_) / 2;
                    const uint32_t col0 = (batch == 0 ? 0u : Cfg::kTmemU) + static_cast<uint32_t>(ncols * ch);
                    uint32_t x[kMaxBlk][16];
#pragma unroll
                    for (int cb = 0; cb < kMaxBlk; ++cb)
                        if (cb * 32 < ncols) tmem_ld_16x256b_x4(acc + ((32u * qd) << 16) + col0 + 32 * cb, x[cb]);
                    tmem_wait_ld();
                    __nv_bfloat16* base = (batch == 0 ? p.w + t.b * p.w_sb + t.t0 * p.w_st + t.hv * p.w_sh
                                                      : p.u + t.b * p.u_sb + t.t0 * p.u_st + t.hv * p.u_sh) +
                                          ncols * ch;
                    const int64_t rs = batch == 0 ? p.w_st : p.u_st;
#pragma unroll
                    for (int cb = 0; cb < kMaxBlk; ++cb) {
                        if (cb * 32 >= ncols) continue;
#pragma unroll
                        for (int half = 0; half < 2; ++half) {
                            uint32_t q4[4];
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj)
                                q4[jj] = pack_bf16x2(__uint_as_float(x[cb][4 * jj + 2 * half]),
                                                     __uint_as_float(x[cb][4 * jj + 2 * half + 1]));
                            quad_transpose(q4, lane);
                            const int row = half ? rb : ra;
                            if (half ? live_b : live_a)
                                *reinterpret_cast<uint4*>(base + row * rs + 32 * cb + 8 * qi) =
                                    make_uint4(q4[0], q4[1], q4[2], q4[3]);
                        }
                    }
                }
            }
        }
        if (issuer) {
            // every MMA this warp issued has completed before TMEM is released
            if (elect_one_sync()) tc_commit(&mma_drain[grp]);
            __syncwarp();
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            mbar_wait(&mma_drain[grp], 0, drain, 0x20);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace cgdr
