// Recurrence and chunk output in one tcgen05 kernel (sm_100a): the hidden-state
// recurrence of kernel_tc.cuh with the chunk output of kernel_chunk_o.cuh
// computed from the state while it is still on chip.  h and v_new never go
// to global memory.  This is the composition of the reference's stage 2 and
// stage 3 (ref/chunk_gated_delta_rule/tests/pytest/chunk_gated_delta_rule_benchmark.py
// :77-79, :129 and :145-175) inside one task loop.
//
// One CTA owns one (sequence, value head) with all VT (64 or 128) value
// columns, K = 128.  Per chunk c (S = state before the chunk, bf16 copy in
// shared memory; scale_i = scale * exp(g_i)):
//   MMA1  [D1; O1] = [w_c; q_c] . S       M=128 N=VT K=128   one MMA for both
//   MMA4  [- ; A ] = [w_c; q_c] . k_c^T   M=128 N=64 K=128   (the w rows are unused)
//   epi1  v_new = u - D1; v_dec = v_new * gate -> in place of u; bf16(v_new) -> vn
//   epiP  P = bf16(bf16(A) * scale * exp(g_i - g_j)), j <= i, else 0 -> over the [w;q] tile
//   MMA2  D2 = k_c^T . v_dec                 M=128 N=VT K=64
//   MMA5  O2 = P . vn                         M=64  N=VT K=64    (over D1: lanes 0-15 of each quadrant)
//   epi2  S = S * alpha + D2 -> bf16 S tile
//   epiO  o = scale_i * O1 + O2 -> bf16 -> TMA store
// The A operand of MMA1/MMA4 interleaves w and q in 16-row groups: rows
// 32j..32j+15 are w rows 16j.., rows 32j+16..32j+31 are q rows 16j...  With
// M=128 (row r in TMEM lane r) each 32-lane quadrant j then holds the w rows
// 16j..16j+15 in its first 16 lanes, where an M=64 accumulator keeps them and
// where the recurrence's epilogue reads D1, and the q rows in its last 16
// lanes.  q . S costs no tensor-core time beyond the M=64 product it rides
// along with (an M=128 N=VT step takes as long as an M=64 one).
//
// The critical chain is the recurrence's (MMA1, epi1, MMA2, epi2); the
// output work (MMA4, epiP, MMA5, epiO) fills the epilogue's waits for the
// tensor cores.  D1/O1/O2 are double-buffered in TMEM so MMA1 of chunk c+1
// never waits for the output of chunk c.
//
// Warp roles (block = 32 * (4*EW + 2), EW = VT/64):
//   warps 0 .. 4*EW-1  epilogue: TMEM quadrant w%4, 64-column slice w/4;
//   warp 4*EW          TMA producer (k_c, w_c, q_c, u_c and the gate inputs);
//   warp 4*EW+1        MMA issuer and TMEM owner.
// Every wait is bounded; on expiry the CTA records the role in the status
// word, drains its own copies and MMAs and returns.
#pragma once

#include "common.cuh"
#include "kernel_tc.cuh"
#include "ptx.cuh"

namespace cgdr {

struct HoMaps {
    CUtensorMap k;  // dims (K, HK, T, B), box (64, 1, 64, 1)
    CUtensorMap w;  // dims (K, H, T, B),  box (64, 1, 16, 1)
    CUtensorMap q;  // dims (K, HK, T, B), box (64, 1, 16, 1)
    CUtensorMap u;  // dims (V, H, T, B),  box (64, 1, 64, 1)
    CUtensorMap o;  // dims (V, H, T, B),  box (64, 1, 16, 1)   (store)
};

struct HoExtra {
    __nv_bfloat16* o;  // [B, T, H, V] (partial varlen chunks are stored element-wise)
    int64_t o_sb, o_st, o_sh;
    float scale;
};

struct HoArgs {
    HoMaps maps;
    FwdHParams p;
    HoExtra x;
};

template <int VT>
struct HoConfig {
    static_assert(VT == 64 || VT == 128, "fused recurrence + output: V in {64, 128}");
    static constexpr int kK = 128;
    static constexpr int EW = VT / 64;
    static constexpr int kEpiWarps = 4 * EW;
    static constexpr int kThreads = 32 * (kEpiWarps + 2);
    static constexpr int kProducerWarp = kEpiWarps;
    static constexpr int kMmaWarp = kEpiWarps + 1;
    static constexpr int kStages = 2;
    static constexpr int kSubV = VT / 64;
    static constexpr int kTileK = 2 * 8192;             // k_c: [64 tokens][128] as two 64-column sub-tiles
    static constexpr int kWQSub = 16384;                // [w;q] 64-column sub-tile: 128 rows x 128 B
    static constexpr int kTileWQ = 2 * kWQSub;
    static constexpr int kTileU = VT * 128;             // [64 tokens][VT]
    static constexpr int kOffK = 0;                     // offsets within a stage
    static constexpr int kOffWQ = kTileK;
    static constexpr int kOffU = kTileK + kTileWQ;
    static constexpr int kStageBytes = kTileK + kTileWQ + kTileU;
    static constexpr int kOffS = kStages * kStageBytes;
    static constexpr int kSSubBytes = kK * 128;         // one 64-column sub-tile of S
    static constexpr int kOffVn = kOffS + kSubV * kSSubBytes;
    static constexpr int kOffOut = kOffVn + kTileU;
    static constexpr int kOffG = kOffOut + kTileU;      // [kStages][64] fp32 gate inputs
    static constexpr int kOffBar = kOffG + kStages * 64 * 4;
    static constexpr int kNumBars = 2 * kStages + 10;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    // TMEM columns: D1/O1/O2 double-buffered at 0 and VT, D2 at 2VT, A at 3VT.
    static constexpr uint32_t kTmemCols = VT == 128 ? 512 : 256;
    static constexpr uint32_t kColD2 = 2 * VT;
    static constexpr uint32_t kColA = 3 * VT;
    static constexpr uint32_t kIdesc1 = umma_idesc_bf16(128, VT, false, true);
    static constexpr uint32_t kIdesc4 = umma_idesc_bf16(128, 64, false, false);
    static constexpr uint32_t kIdesc2 = umma_idesc_bf16(kK, VT, true, true);
    static constexpr uint32_t kIdesc5 = umma_idesc_bf16(64, VT, false, true);
};

template <int VT>
__global__ void __launch_bounds__(HoConfig<VT>::kThreads, 1) fwd_ho_tc_kernel(const __grid_constant__ HoArgs args)
{
    using Cfg = HoConfig<VT>;
    const FwdHParams& p = args.p;
    const HoExtra& x = args.x;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;
    uint64_t* empty = bars + Cfg::kStages;
    uint64_t* mma1_done = bars + 2 * Cfg::kStages;
    uint64_t* mma4_done = mma1_done + 1;
    uint64_t* mma2_done = mma1_done + 2;
    uint64_t* mma5_done = mma1_done + 3;
    uint64_t* vdec_ready = mma1_done + 4;
    uint64_t* s_ready = mma1_done + 5;
    uint64_t* p_ready = mma1_done + 6;
    uint64_t* o_free = mma1_done + 7;  // [2]
    uint64_t* mma_drain = mma1_done + 9;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* never_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (p.status && (*reinterpret_cast<volatile int*>(p.status) & 0x2)) return;  // bad varlen metadata

    int64_t n, hv;
    {
        const int64_t bid = blockIdx.x;
        hv = bid % p.H;
        const int64_t rank = bid / p.H;
        n = (p.varlen && p.seq_order) ? p.seq_order[rank] : rank;
    }
    const SeqInfo si = seq_info(p, n);
    const int64_t kh = hv / (p.H / p.HK);
    const int64_t nchunks = (si.len + kChunk - 1) / kChunk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full[s], 1 + 32);  // TMA bytes + 32 cp.async arrivals (gate inputs)
            mbar_init(&empty[s], 1);
        }
        mbar_init(mma1_done, 1);
        mbar_init(mma4_done, 1);
        mbar_init(mma2_done, 1);
        mbar_init(mma5_done, 1);
        mbar_init(vdec_ready, Cfg::kEpiWarps);
        mbar_init(s_ready, Cfg::kEpiWarps);
        mbar_init(p_ready, Cfg::kEpiWarps);
        mbar_init(&o_free[0], Cfg::kEpiWarps);
        mbar_init(&o_free[1], Cfg::kEpiWarps);
        mbar_init(mma_drain, 1);
        *abort_flag = 0;
        *never_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == Cfg::kMmaWarp) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == Cfg::kProducerWarp && lane == 0) {
        prefetch_tensormap(&args.maps.k);
        prefetch_tensormap(&args.maps.w);
        prefetch_tensormap(&args.maps.q);
        prefetch_tensormap(&args.maps.u);
        prefetch_tensormap(&args.maps.o);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const WaitCtl ctl{abort_flag, p.status, p.timeout_ns};
    const uint32_t sbase = smem_u32(smem);

    auto k_addr = [&](int s) { return sbase + s * Cfg::kStageBytes + Cfg::kOffK; };
    auto wq_addr = [&](int s) { return sbase + s * Cfg::kStageBytes + Cfg::kOffWQ; };
    auto u_addr = [&](int s) { return sbase + s * Cfg::kStageBytes + Cfg::kOffU; };

    if (warp == Cfg::kProducerWarp) {
        // ------------------------------------------------------------ producer
        int64_t issued = 0;
        const int64_t gbase = si.b * p.g_sb + hv * p.g_sh;
        for (int64_t c = 0; c < nchunks; ++c) {
            const int s = static_cast<int>(c % Cfg::kStages);
            const uint32_t use = static_cast<uint32_t>(c / Cfg::kStages);
            bool go = true;
            if (c >= Cfg::kStages && lane == 0) go = mbar_wait(&empty[s], (use - 1) & 1, ctl, 0x10);
            if (p.fault_inject && c == 1) go = false;  // test hook: consumers' waits must expire
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (!go) break;
            const int t0 = static_cast<int>(si.bos + c * kChunk);
            if (lane == 0) {
                uint8_t* st = smem + s * Cfg::kStageBytes;
                const int b = static_cast<int>(si.b);
                mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
#pragma unroll
                for (int sub = 0; sub < 2; ++sub) {
                    tma_load_4d(&args.maps.k, st + Cfg::kOffK + sub * 8192, &full[s], sub * 64, static_cast<int>(kh),
                                t0, b);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint8_t* grp = st + Cfg::kOffWQ + sub * Cfg::kWQSub + j * 4096;
                        tma_load_4d(&args.maps.w, grp, &full[s], sub * 64, static_cast<int>(hv), t0 + 16 * j, b);
                        tma_load_4d(&args.maps.q, grp + 2048, &full[s], sub * 64, static_cast<int>(kh), t0 + 16 * j, b);
                    }
                }
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubV; ++sub)
                    tma_load_4d(&args.maps.u, st + Cfg::kOffU + sub * 8192, &full[s], sub * 64, static_cast<int>(hv),
                                t0, b);
            }
            if (p.g) {
                const int len = static_cast<int>(si.len - c * kChunk < kChunk ? si.len - c * kChunk : kChunk);
                float* gs = reinterpret_cast<float*>(smem + Cfg::kOffG) + 64 * s;
                if (lane < len) cp_async_4(gs + lane, p.g + gbase + (t0 + lane) * p.g_st);
                if (lane + 32 < len) cp_async_4(gs + lane + 32, p.g + gbase + (t0 + lane + 32) * p.g_st);
            }
            cp_async_arrive_noinc(&full[s]);
            ++issued;
        }
        if (lane == 0) {
            const int64_t first = issued > Cfg::kStages ? issued - Cfg::kStages : 0;
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            for (int64_t c = first; c < issued; ++c)
                mbar_wait(&full[c % Cfg::kStages], static_cast<uint32_t>(c / Cfg::kStages) & 1, drain, 0x10);
        }
    } else if (warp == Cfg::kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        auto wait_warp = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, ctl, 0x20) ? 1 : 0) != 0;
        };
        const uint32_t s_addr = sbase + Cfg::kOffS;
        const uint32_t vn_addr = sbase + Cfg::kOffVn;
        for (int64_t c = 0; c < nchunks; ++c) {
            const int s = static_cast<int>(c % Cfg::kStages);
            const int bsel = static_cast<int>(c & 1);
            const uint32_t d1 = tmem + static_cast<uint32_t>(bsel * VT);
            if (!wait_warp(&full[s], static_cast<uint32_t>(c / Cfg::kStages) & 1)) break;
            if (!wait_warp(s_ready, static_cast<uint32_t>(c) & 1)) break;
            if (c >= 2 && !wait_warp(&o_free[bsel], static_cast<uint32_t>(c / 2 - 1) & 1)) break;
            tc_fence_after();
            const uint64_t awq = umma_desc_sw128(wq_addr(s), 16, 1024);
            const uint64_t bs = umma_desc_sw128(s_addr, Cfg::kSSubBytes, 1024);
            const uint64_t bk = umma_desc_sw128(k_addr(s), 16, 1024);
            if (elect_one_sync()) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    tc_mma_bf16(d1, awq + static_cast<uint64_t>(((kk >> 2) * Cfg::kWQSub + (kk & 3) * 32) >> 4),
                                bs + static_cast<uint64_t>((kk * 2048) >> 4), Cfg::kIdesc1, kk > 0 ? 1u : 0u);
                tc_commit(mma1_done);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    tc_mma_bf16(tmem + Cfg::kColA,
                                awq + static_cast<uint64_t>(((kk >> 2) * Cfg::kWQSub + (kk & 3) * 32) >> 4),
                                bk + static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4), Cfg::kIdesc4,
                                kk > 0 ? 1u : 0u);
                tc_commit(mma4_done);
            }
            __syncwarp();
            if (!wait_warp(vdec_ready, static_cast<uint32_t>(c) & 1)) break;
            tc_fence_after();
            const uint64_t a2 = umma_desc_sw128(k_addr(s), 8192, 1024);
            const uint64_t b2 = umma_desc_sw128(u_addr(s), 8192, 1024);
            if (elect_one_sync()) {
#pragma unroll
                for (int tt = 0; tt < 4; ++tt)
                    tc_mma_bf16(tmem + Cfg::kColD2, a2 + static_cast<uint64_t>((tt * 2048) >> 4),
                                b2 + static_cast<uint64_t>((tt * 2048) >> 4), Cfg::kIdesc2, tt > 0 ? 1u : 0u);
                tc_commit(mma2_done);
            }
            __syncwarp();
            if (!wait_warp(p_ready, static_cast<uint32_t>(c) & 1)) break;
            tc_fence_after();
            const uint64_t pa = umma_desc_sw128(wq_addr(s), 16, 1024);  // P over the first [w;q] rows
            const uint64_t vb = umma_desc_sw128(vn_addr, 8192, 1024);
            if (elect_one_sync()) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc_mma_bf16(d1, pa + static_cast<uint64_t>((kk * 32) >> 4), vb + static_cast<uint64_t>((kk * 2048) >> 4),
                                Cfg::kIdesc5, kk > 0 ? 1u : 0u);
                tc_commit(mma5_done);
                tc_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (elect_one_sync()) tc_commit(mma_drain);
        __syncwarp();
        WaitCtl drain{never_flag, p.status, p.timeout_ns};
        mbar_wait(mma_drain, 0, drain, 0x20);
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;           // TMEM lane quadrant: token rows 16q..16q+15
        const int e = warp >> 2;          // 64-column slice
        const int cbase = 64 * e;
        uint8_t* s_tile = smem + Cfg::kOffS;
        uint8_t* vn_tile = smem + Cfg::kOffVn;
        uint8_t* out_tile = smem + Cfg::kOffOut;
        const int ta = 16 * q + (lane >> 2);  // epi1 token rows ta, ta+8
        const int tb = ta + 8;
        const int pc = 2 * (lane & 3);
        const int orow = 16 * q + (lane & 15);  // epiP / epiO: one token row per lane pair (lane, lane^16)
        const int ohalf = lane >> 4;            // epiO: column half of the slice this lane stores
        const float sc = x.scale;

        // state rows owned by this thread: row 32q+lane, columns cbase..cbase+63
        float st[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            float v = 0.0f;
            if (p.h0)
                v = load_io(p.h0, p.h0_dtype,
                            si.n * p.h0_sn + hv * p.h0_sh + (32 * q + lane) * p.h0_sk + (cbase + i) * p.h0_sv);
            st[i] = v;
        }
        auto write_state_tile = [&]() {
            const int row = 32 * q + lane;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint4 v;
                v.x = pack_bf16x2(st[8 * j + 0], st[8 * j + 1]);
                v.y = pack_bf16x2(st[8 * j + 2], st[8 * j + 3]);
                v.z = pack_bf16x2(st[8 * j + 4], st[8 * j + 5]);
                v.w = pack_bf16x2(st[8 * j + 6], st[8 * j + 7]);
                *reinterpret_cast<uint4*>(s_tile + sw128_off(row, cbase + 8 * j, Cfg::kSSubBytes)) = v;
            }
        };

        // swizzled byte offsets of this thread's (row, column pair) elements in the u / v_decay /
        // v_new tiles (the same every chunk)
        uint32_t offs[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
            offs[i] = sw128_off(half ? tb : ta, cbase + 32 * cb + 8 * j + pc, 8192);
        }

        bool ok = true;
        write_state_tile();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_ready);

        for (int64_t c = 0; c < nchunks && ok; ++c) {
            const int s = static_cast<int>(c % Cfg::kStages);
            const int bsel = static_cast<int>(c & 1);
            const uint32_t d1col = static_cast<uint32_t>(bsel * VT);
            const int64_t t0 = si.bos + c * kChunk;
            const int len = static_cast<int>(si.len - c * kChunk < kChunk ? si.len - c * kChunk : kChunk);
            uint8_t* stage = smem + s * Cfg::kStageBytes;

            // ================= epilogue 1: v_new, v_decay =================
            if (!mbar_wait(&full[s], static_cast<uint32_t>(c / Cfg::kStages) & 1, ctl, 0x40)) { ok = false; break; }
            const float* gs = reinterpret_cast<const float*>(smem + Cfg::kOffG) + 64 * s;
            float g_l = 0.f, g_a = 0.f, g_b = 0.f;
            if (p.g) {
                g_l = gs[len - 1];
                g_a = ta < len ? gs[ta] : g_l;
                g_b = tb < len ? gs[tb] : g_l;
            }
            float gate_a = 1.0f, gate_b = 1.0f, alpha = 1.0f;
            if (p.use_g) {
                gate_a = safe_exp(g_l - g_a);
                gate_b = safe_exp(g_l - g_b);
                alpha = expf(g_l);
            }
            uint8_t* ut = stage + Cfg::kOffU;
            uint32_t uraw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) uraw[i] = *reinterpret_cast<const uint32_t*>(ut + offs[i]);
            if (!mbar_wait(mma1_done, static_cast<uint32_t>(c) & 1, ctl, 0x40)) { ok = false; break; }
            tc_fence_after();
            uint32_t acc[2][16];
#pragma unroll
            for (int cb = 0; cb < 2; ++cb)
                tmem_ld_16x256b_x4(tmem + ((32u * q) << 16) + d1col + static_cast<uint32_t>(cbase + 32 * cb), acc[cb]);
            tmem_wait_ld();
            uint32_t vds[16], vns[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                const float gt = half ? gate_b : gate_a;
                const float2 uu = unpack_bf16x2(uraw[i]);
                const float n0 = uu.x - __uint_as_float(acc[cb][4 * j + 2 * half + 0]);
                const float n1 = uu.y - __uint_as_float(acc[cb][4 * j + 2 * half + 1]);
                const bool valid = (half ? tb : ta) < len;
                vds[i] = valid ? pack_bf16x2(n0 * gt, n1 * gt) : 0u;
                vns[i] = valid ? pack_bf16x2(n0, n1) : 0u;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) *reinterpret_cast<uint32_t*>(ut + offs[i]) = vds[i];
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(vdec_ready);
            // bf16 v_new: the B operand of MMA5 (MMA5 of chunk c-1 completed before mma1_done(c))
#pragma unroll
            for (int i = 0; i < 16; ++i) *reinterpret_cast<uint32_t*>(vn_tile + offs[i]) = vns[i];

            // ================= P from A = q . k^T =================
            // lanes 16..31 hold the q rows of the M=128 accumulator: row orow, columns of this warp
            if (!mbar_wait(mma4_done, static_cast<uint32_t>(c) & 1, ctl, 0x40)) { ok = false; break; }
            tc_fence_after();
            // scale * exp(g_i) of the output row: read now, while the stage's gate inputs are
            // still this chunk's (the producer refills the stage once MMA5 has completed)
            const float g_i = (p.g && orow < len) ? gs[orow] : 0.0f;
            const float f_o = __fmul_rn(sc, expf(g_i));
            {
                // Lanes 16..31 hold the q rows of A; each 16-column block is split so that the
                // lane pair (l, l^16), which shares row orow, computes 8 columns each: lanes
                // 16..31 columns 0..7 of the block, lanes 0..15 columns 8..15 (one shuffle).
                constexpr int kPCols = 64 / Cfg::EW;  // A columns per warp
                const int pbase = kPCols * e;
                const int half8 = lane < 16 ? 8 : 0;
#pragma unroll
                for (int blk = 0; blk < kPCols / 16; ++blk) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(tmem + ((32u * q) << 16) + Cfg::kColA + static_cast<uint32_t>(pbase + 16 * blk), r);
                    tmem_wait_ld();
                    uint32_t a[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint32_t other = __shfl_xor_sync(0xffffffffu, r[8 + i], 16);
                        a[i] = lane < 16 ? other : r[i];
                    }
                    const int j0 = pbase + 16 * blk + half8;  // first of this lane's 8 columns
                    float gj[8];
                    {
                        const float4 g0 = *reinterpret_cast<const float4*>(gs + j0);
                        const float4 g1 = *reinterpret_cast<const float4*>(gs + j0 + 4);
                        gj[0] = g0.x; gj[1] = g0.y; gj[2] = g0.z; gj[3] = g0.w;
                        gj[4] = g1.x; gj[5] = g1.y; gj[6] = g1.z; gj[7] = g1.w;
                    }
                    uint32_t pk[4];
#pragma unroll
                    for (int i = 0; i < 8; i += 2) {
                        // bf16(A) for the pair in one conversion
                        const float2 sb = unpack_bf16x2(pack_bf16x2(__uint_as_float(a[i]), __uint_as_float(a[i + 1])));
                        const int j = j0 + i;
                        const float e0 = __expf(g_i - ((p.g && j < len) ? gj[i] : 0.0f));
                        const float e1 = __expf(g_i - ((p.g && j + 1 < len) ? gj[i + 1] : 0.0f));
                        const float x0 = (j <= orow) ? __fmul_rn(__fmul_rn(sb.x, sc), e0) : 0.0f;
                        const float x1 = (j + 1 <= orow) ? __fmul_rn(__fmul_rn(sb.y, sc), e1) : 0.0f;
                        pk[i / 2] = pack_bf16x2(x0, x1);
                    }
                    uint8_t* prow = stage + Cfg::kOffWQ + orow * 128;
                    *reinterpret_cast<uint4*>(prow + ((((j0 >> 3)) ^ (orow & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_ready);

            // ================= epilogue 2: state =================
            if (!mbar_wait(mma2_done, static_cast<uint32_t>(c) & 1, ctl, 0x40)) { ok = false; break; }
            tc_fence_after();
            const bool more = c + 1 < nchunks;
            {
                const uint32_t ta2 = tmem + Cfg::kColD2 + ((32u * q) << 16) + static_cast<uint32_t>(cbase);
#pragma unroll
                for (int cb = 0; cb < 2; ++cb) {
                    uint32_t r[2][16];
                    tmem_ld_32x32b_x16(ta2 + 32 * cb, r[0]);
                    tmem_ld_32x32b_x16(ta2 + 32 * cb + 16, r[1]);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 2; ++j)
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float& sv = st[32 * cb + 16 * j + i];
                            sv = fmaf(sv, alpha, __uint_as_float(r[j][i]));
                        }
                }
            }
            if (more) {
                write_state_tile();
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_ready);
            } else {
                tc_fence_before();
            }

            // ================= output =================
            if (!mbar_wait(mma5_done, static_cast<uint32_t>(c) & 1, ctl, 0x40)) { ok = false; break; }
            tc_fence_after();
            uint32_t ov[32];  // this lane's row orow, columns cbase + 32*ohalf ..
            {
                // lanes 0..15 hold O2 (rows 16q+lane), lanes 16..31 O1 (rows 16q+lane-16), all 64
                // columns of the slice; lanes 0..15 store columns 0..31 and lanes 16..31 columns
                // 32..63, so each lane sends its partner exactly the half the partner stores
                uint32_t r[4][16];
                const uint32_t base = tmem + ((32u * q) << 16) + d1col + static_cast<uint32_t>(cbase);
#pragma unroll
                for (int m = 0; m < 4; ++m) tmem_ld_32x32b_x16(base + 16 * m, r[m]);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const uint32_t lo = r[i >> 4][i & 15], hi = r[2 + (i >> 4)][i & 15];
                    // lane < 16 sends O2 columns 32+i, receives O1 columns i; lane >= 16 sends O1
                    // columns i, receives O2 columns 32+i
                    const float got = __uint_as_float(__shfl_xor_sync(0xffffffffu, ohalf ? lo : hi, 16));
                    const float o1 = ohalf ? __uint_as_float(hi) : got;
                    const float o2 = ohalf ? got : __uint_as_float(lo);
                    ov[i] = __float_as_uint(fmaf(f_o, o1, o2));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[bsel]);
            const bool partial_varlen = p.varlen && len < kChunk;
            if (partial_varlen) {
                if (orow < len) {
                    __nv_bfloat16* dst = x.o + si.b * x.o_sb + (t0 + orow) * x.o_st + hv * x.o_sh + cbase + 32 * ohalf;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        reinterpret_cast<uint4*>(dst)[j] = make_uint4(
                            pack_bf16x2(__uint_as_float(ov[8 * j + 0]), __uint_as_float(ov[8 * j + 1])),
                            pack_bf16x2(__uint_as_float(ov[8 * j + 2]), __uint_as_float(ov[8 * j + 3])),
                            pack_bf16x2(__uint_as_float(ov[8 * j + 4]), __uint_as_float(ov[8 * j + 5])),
                            pack_bf16x2(__uint_as_float(ov[8 * j + 6]), __uint_as_float(ov[8 * j + 7])));
                }
            } else {
                // staging rows of this warp are free once its previous store has read them
                if (lane == 0) bulk_wait_group_read0();
                __syncwarp();
                uint8_t* srow = out_tile + e * 8192 + orow * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(srow + (((4 * ohalf + j) ^ (orow & 7)) << 4)) = make_uint4(
                        pack_bf16x2(__uint_as_float(ov[8 * j + 0]), __uint_as_float(ov[8 * j + 1])),
                        pack_bf16x2(__uint_as_float(ov[8 * j + 2]), __uint_as_float(ov[8 * j + 3])),
                        pack_bf16x2(__uint_as_float(ov[8 * j + 4]), __uint_as_float(ov[8 * j + 5])),
                        pack_bf16x2(__uint_as_float(ov[8 * j + 6]), __uint_as_float(ov[8 * j + 7])));
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_4d(&args.maps.o, out_tile + e * 8192 + 16 * q * 128, cbase, static_cast<int>(hv),
                                 static_cast<int>(t0 + 16 * q), static_cast<int>(si.b));
                    bulk_commit_group();
                }
            }
        }
        // ---- final state (plain stores; once per task)
        if (ok && p.final_state) {
#pragma unroll
            for (int i = 0; i < 64; ++i)
                store_io(p.final_state, p.f_dtype,
                         si.n * p.f_sn + hv * p.f_sh + (32 * q + lane) * p.f_sk + (cbase + i) * p.f_sv, st[i]);
        }
        if (lane == 0) bulk_wait_group0();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == Cfg::kMmaWarp) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace cgdr
