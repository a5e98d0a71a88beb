// Tensor-core (tcgen05) kernel for sm_100a.
//
// One CTA owns one (sequence, value head, V tile of VT columns) and walks the
// sequence's 64-token chunks in order -- the task split of the reference's
// ProcessTask (op_kernel/chunk_gated_delta_rule_fwd_h.h:421-510), with the
// state resident on chip instead of bounced through global memory.
//
// Warp roles (block = 32 * (4*EW + 1 + chains) threads):
//   warps 0 .. 4*EW-1  epilogue: warp w reads TMEM lane quadrant w%4 and the
//                      column slice (w/4) of width VT/EW;
//   warp 4*EW          TMA producer: k_c, w_c, u_c of chunk c into a ring of
//                      STAGES shared-memory stages;
//   warp 4*EW+1 (+c)   MMA issuer of chain c; the first one owns TMEM.
// Usually the CTA's VT columns are one chain.  With CH = 2 (K tile 128, VT = 32 or
// 128, EW = 2) each column slice of VT / 2 is a chain of its own: its own MMAs
// (N = VT / 2), TMEM accumulators, state sub-tile and barriers, with only the load
// stages shared, so that one chain's epilogues run while the other's MMAs do.
//
// Per chunk c (S = state before the chunk, bf16 copy in shared memory):
//   MMA1  D1[t,v] = sum_k w_c[t,k] S[k,v]        M=64, N=VT, K=K   (A K-major, B MN-major)
//   epi1  v_new = u - D1 -> v_new tile (TMA store); v_dec = v_new*gate -> in place of u
//   MMA2  D2[k,v] = sum_t k_c[t,k] v_dec[t,v]    M=K,  N=VT, K=64  (A, B MN-major)
//   epi2  S = S*alpha + D2 (fp32 registers) -> bf16 S tile -> h[c+1] (TMA store)
// The shared-memory tiles use the 128-byte swizzle in 64-column (128 B) sub-tiles,
// or (32-column tiles) the 64-byte swizzle, or (two 16-column chains) the 32-byte
// swizzle in 16-column sub-tiles, so one layout serves the TMA boxes and the UMMA
// descriptors.
//
// The K tile K_ is 64, 128 or 256; a caller's K below it arrives zero-filled from
// the tensor maps (rows past K of the state stay zero and are never stored).  With
// K_ = 256, MMA2 runs as two M = 128 halves into separate TMEM column ranges and
// epilogue warp w owns state rows 128 (w / 4) + 32 (w % 4) + lane.  Warps whose
// column slice is narrower than a 64-column sub-tile stage v_new in regions of
// their own (kSplitVout); with the reference arithmetic's sixteen-warp 128-column
// tiles the h store of a sub-tile is shared by two warps (kSharedH).
//
// Every wait is bounded (WaitCtl); on expiry the CTA raises its abort flag,
// records the role in the status word, drains its own copies and returns.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace cgdr {

struct TcMaps {
    CUtensorMap k;  // dims (K, HK, T, B), box (64, 1, 64, 1)
    CUtensorMap w;  // dims (K, H, T, B),  box (64, 1, 64, 1)
    CUtensorMap u;  // dims (V, H, T, B),  box (64, 1, 64, 1)
    CUtensorMap v;  // dims (V, H, T, B),  box (64, 1, 16, 1)   (v_new store, 16 token rows)
    CUtensorMap h;  // dims (V, K, H, NTdim, B), box (64, ROWS, 1, 1, 1)
};

struct TcArgs {
    TcMaps maps;
    FwdHParams p;
};

template <int K_, int VT, int STAGES, int EW, int CH = 1>
struct TcConfig {
    static_assert(K_ == 64 || K_ == 128 || K_ == 256, "tensor-core path: K tile in {64, 128, 256}");
    static_assert(VT == 32 || VT == 64 || VT == 128, "tensor-core path: V tile in {32, 64, 128}");
    static_assert(EW == 1 || EW == VT / 64 || (K_ == 256 && VT == 64 && EW == 2) || (K_ == 128 && VT == 128 && EW == 4) ||
                      (K_ == 128 && VT == 32 && EW == 2 && CH == 2),
                  "column split must be 1, one warp per 64-column sub-tile, (K = 256) two 32-column halves, "
                  "(K = 128, VT = 128) four 32-column quarters or (K = 128, VT = 32) two 16-column chains");
    static_assert(CH == 1 || (CH == 2 && EW == 2 && K_ == 128 && (VT == 32 || VT == 128)),
                  "two chains per CTA: K tile 128, VT 32 or 128, one column slice each");
    static_assert(VT != 32 || K_ == 128, "32-column tiles: K = 128");
    static_assert(K_ != 256 || VT == 64, "K = 256: 64-column tiles");
    // each column slice a chain of its own (CH = 2), or one chain
    static constexpr int kChains = CH;
    // Swizzle of the u_c / v_new / S tiles: the two 16-column chains keep them in
    // 16-column sub-tiles of 32-byte rows, 32-column tiles in 64-byte rows, wider
    // tiles in 64-column sub-tiles of 128-byte rows.
    static constexpr int kSwz = VT == 32 ? (kChains == 2 ? 32 : 64) : 128;
    static constexpr int kRowB = kSwz;                  // bytes per row of a u_c / v_new / S sub-tile
    static constexpr int kSubCols = kSwz / 2;           // columns per sub-tile
    static constexpr int kUSub = 64 * kRowB;            // one sub-tile of u_c / v_new (64 token rows)
    static constexpr int kEpiWarps = 4 * EW;
    static constexpr int kThreads = 32 * (kEpiWarps + 1 + kChains);
    static constexpr int kProducerWarp = kEpiWarps;
    static constexpr int kMmaWarp = kEpiWarps + 1;      // chain c's MMA issuer: kMmaWarp + c
    static constexpr int kCW = VT / EW;                 // columns per epilogue warp
    static constexpr int kChainCols = VT / kChains;     // columns of one chain (N of its MMAs)
    static constexpr int kSubK = K_ / 64;              // 64-column sub-tiles of k_c / w_c
    static constexpr int kSubV = VT / kSubCols;         // sub-tiles of u_c / S / v_new
    static constexpr int kTileKBytes = K_ * 128;       // [64 tokens][K] bf16
    static constexpr int kTileUBytes = VT * 128;       // [64 tokens][VT] bf16
    static constexpr int kStageBytes = 2 * kTileKBytes + kTileUBytes;
    static constexpr int kSBytes = K_ * VT * 2;        // [K][VT] bf16
    static constexpr int kSSubBytes = K_ * kRowB;      // one sub-tile of S
    static constexpr int kVoutBytes = 64 * VT * 2;
    static constexpr int kOffS = STAGES * kStageBytes;
    static constexpr int kOffVout = kOffS + kSBytes;
    static constexpr int kOffG = kOffVout + kVoutBytes;  // [STAGES][64] fp32 gate inputs
    static constexpr int kOffBar = kOffG + STAGES * 64 * 4;
    // full/empty per stage; per chain mma1_done, mma2_done, drain, s_ready, vdec_ready; h_read[4]
    static constexpr int kNumBars = 2 * STAGES + 5 * kChains + 4;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + tmem slot, abort flag, alignment
    static constexpr uint32_t kStageTx = kStageBytes;
    // MMA2 (M = K) as M = 128 halves when K = 256: D2 rows [128 m, 128 m + 128) at TMEM
    // columns [VT (1 + m), VT (2 + m)).  D1 at [0, VT).
    static constexpr int kM2 = K_ == 256 ? 128 : K_;
    static constexpr int kM2Halves = K_ / kM2;
    static constexpr int kTmemUsed = VT * (1 + kM2Halves);
    static constexpr int kTmemCols = kTmemUsed <= 32 ? 32 : kTmemUsed <= 64 ? 64 : kTmemUsed <= 128 ? 128
                                     : kTmemUsed <= 256 ? 256 : 512;
    static constexpr int kHRows = (K_ == 64) ? 16 : 32;  // S rows per warp quadrant (h store box)
    // Epilogue 2 (K >= 128): each thread owns one state row and kE2Cols of its columns.
    // K = 256: warp w holds rows 128 (w / 4) + 32 (w % 4) + lane, all VT columns;
    // K = 128: rows 32 (w % 4) + lane, the warp's epilogue-1 column slice.
    static constexpr int kE2Cols = K_ == 256 ? VT : kCW;
    // Epilogue-1 column slices narrower than a 64-column sub-tile (K = 256): each warp
    // stages its v_new rows in a region of its own, 32 columns of 64-byte rows with the
    // 64-byte swizzle, and stores it with a 32-column box, so no two warps share a store.
    static constexpr bool kSplitVout = kCW < kSubCols;
    // Epilogue-2 column slices narrower than a 64-column sub-tile (K = 128 with four
    // 32-column quarters): the quadrant's warps at even slices store h for their
    // sub-tile once every epilogue warp wrote its part (s_ready), and the odd slices
    // rewrite their half of the state tile only after that store has read it (h_read).
    static constexpr bool kSharedH = K_ >= 128 && kE2Cols < kSubCols;
    static constexpr int kVoutRegion = 64 * 64;  // bytes of one warp's region (64 rows x 64 B)
    static constexpr int kMinBlocks = (VT == 64 && K_ != 256) ? 2 : 1;  // CTAs resident per SM the tile is sized for
    static constexpr uint32_t kIdesc1 = umma_idesc_bf16(64, kChainCols, false, true);
    static constexpr uint32_t kIdesc2 = umma_idesc_bf16(kM2, kChainCols, true, true);
};

// Byte offset of element (row, col) inside a swizzled tile made of 64-column
// sub-tiles of `sub_bytes` each (128-byte rows, 16-byte chunks XOR row%8).
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int sub_bytes)
{
    const int sub = col >> 6, cc = col & 63;
    return sub * sub_bytes + row * 128 + ((((cc >> 3) ^ (row & 7)) & 7) << 4) + ((cc & 7) << 1);
}

// Byte offset of element (row, col) of a u_c / v_new / S tile (SWZ = swizzle bytes):
//   128  64-column sub-tiles of 128-byte rows (sw128_off);
//    64  one 32-column tile of 64-byte rows, 16-byte chunks XORed with (row / 2) % 4;
//    32  16-column sub-tiles of 32-byte rows, 16-byte chunks XORed with (row / 4) % 2.
template <int SWZ>
__device__ __forceinline__ uint32_t tile_off(int row, int col, int sub_bytes)
{
    if constexpr (SWZ == 32)
        return (col >> 4) * sub_bytes + row * 32 + ((((col >> 3) ^ (row >> 2)) & 1) << 4) + ((col & 7) << 1);
    else if constexpr (SWZ == 64)
        return row * 64 + ((((col >> 3) ^ (row >> 1)) & 3) << 4) + ((col & 7) << 1);
    else
        return sw128_off(row, col, sub_bytes);
}

// MN-major operand descriptor of a u_c / v_new / S tile (see tile_off): MN atoms of
// SWZ / 2 columns one sub-tile apart, 8-row groups 8 SWZ bytes apart.
template <int SWZ>
__device__ __forceinline__ uint64_t umma_desc_mn(uint32_t saddr, uint32_t sub_bytes)
{
    if constexpr (SWZ == 32)
        return umma_desc_sw32(saddr, sub_bytes, 256);
    else if constexpr (SWZ == 64)
        return umma_desc_sw64(saddr, sub_bytes, 512);
    else
        return umma_desc_sw128(saddr, sub_bytes, 1024);
}

__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gmem_src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}

// Arrive on `bar` once this thread's earlier cp.async copies have landed; the
// arrival is one of those counted when the barrier was initialised.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Pending-group waits of the bulk (TMA) stores issued by this thread.
__device__ __forceinline__ void bulk_wait_group_read1()
{
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v)
{
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// The epilogue's state values: fp32 for the fp32-state arithmetic or, for the
// reference arithmetic, whose state is bf16 between chunks, bf16 pairs packed two to
// a register (values i, i + 1 with i even share a register: same row, adjacent columns).
template <bool PACKED, int N>
struct StateRegs {
    float f[PACKED ? 1 : N];
    uint32_t b[PACKED ? N / 2 : 1];
    __device__ __forceinline__ float get(int i) const
    {
        if constexpr (PACKED)
            return __uint_as_float((i & 1) ? (b[i >> 1] & 0xffff0000u) : (b[i >> 1] << 16));
        else
            return f[i];
    }
    // bf16 bits of values i, i + 1 (i even)
    __device__ __forceinline__ uint32_t pair_bits(int i) const
    {
        if constexpr (PACKED)
            return b[i >> 1];
        else
            return pack_bf16x2(f[i], f[i + 1]);
    }
    // bf16 bits of values i, i + 1 (i even; packed only)
    __device__ __forceinline__ void set_pair_bits(int i, uint32_t bits) { b[i >> 1] = bits; }
    // values i, i + 1 (i even); rounded to bf16 when packed
    __device__ __forceinline__ void set_pair(int i, float lo, float hi)
    {
        if constexpr (PACKED) {
            b[i >> 1] = pack_bf16x2(lo, hi);
        } else {
            f[i] = lo;
            f[i + 1] = hi;
        }
    }
};

template <int K_, int VT, int STAGES, int EW, bool REF, int CH = 1>
__global__ void __launch_bounds__(TcConfig<K_, VT, STAGES, EW, CH>::kThreads,
                                  TcConfig<K_, VT, STAGES, EW, CH>::kMinBlocks)
    fwd_h_tc_kernel(const __grid_constant__ TcArgs args)
{
    using Cfg = TcConfig<K_, VT, STAGES, EW, CH>;
    const FwdHParams& p = args.p;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // this warp's chain: an MMA issuer's own, an epilogue warp's column slice (two chains)
    const int chain = warp > Cfg::kProducerWarp ? warp - Cfg::kMmaWarp
                                                : (Cfg::kChains == 2 && warp < Cfg::kEpiWarps ? (warp >> 2) : 0);

    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* chain_bars = bars + 2 * STAGES;  // [kChains][5]
    uint64_t* mma1_done = chain_bars + 5 * chain;
    uint64_t* mma2_done = mma1_done + 1;
    uint64_t* mma_drain = mma1_done + 2;
    uint64_t* s_ready = mma1_done + 3;     // every epilogue warp of the chain wrote its part of S
    uint64_t* vdec_ready = mma1_done + 4;  // every epilogue warp of the chain wrote its rows of v_decay
    uint64_t* h_read = chain_bars + 5 * Cfg::kChains;  // per quadrant (kSharedH): the h store read the state tile
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* never_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);  // drains ignore aborts

    if (p.status && (*reinterpret_cast<volatile int*>(p.status) & 0x2)) return;  // bad varlen metadata

    int64_t n, hv, vt;
    {
        const int64_t bid = blockIdx.x;
        vt = bid % p.n_vtiles;
        const int64_t rest = bid / p.n_vtiles;
        hv = rest % p.H;
        const int64_t rank = rest / p.H;
        n = (p.varlen && p.seq_order) ? p.seq_order[rank] : rank;
    }
    const SeqInfo si = seq_info(p, n);
    const int64_t kh = hv / (p.H / p.HK);
    const int v0 = static_cast<int>(vt * VT);
    const int64_t nchunks = (si.len + kChunk - 1) / kChunk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1 + 32);  // TMA bytes + 32 cp.async arrivals (gate inputs)
            mbar_init(&empty[s], Cfg::kChains);  // each chain's MMA2 has read the stage
        }
        for (int c = 0; c < Cfg::kChains; ++c) {
            mbar_init(chain_bars + 5 * c + 0, 1);                              // mma1_done
            mbar_init(chain_bars + 5 * c + 1, 1);                              // mma2_done
            mbar_init(chain_bars + 5 * c + 2, 1);                              // drain
            mbar_init(chain_bars + 5 * c + 3, Cfg::kEpiWarps / Cfg::kChains);  // s_ready
            mbar_init(chain_bars + 5 * c + 4, Cfg::kEpiWarps / Cfg::kChains);  // vdec_ready
        }
        for (int q4 = 0; q4 < 4; ++q4) mbar_init(&h_read[q4], EW / 2 > 0 ? EW / 2 : 1);
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
        prefetch_tensormap(&args.maps.u);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const WaitCtl ctl{abort_flag, p.status, p.timeout_ns};
    const uint32_t sbase = smem_u32(smem);

    auto kc_addr = [&](int s) { return sbase + s * Cfg::kStageBytes; };
    auto wc_addr = [&](int s) { return sbase + s * Cfg::kStageBytes + Cfg::kTileKBytes; };
    auto uc_addr = [&](int s) { return sbase + s * Cfg::kStageBytes + 2 * Cfg::kTileKBytes; };

    if (warp == Cfg::kProducerWarp) {
        // ------------------------------------------------------------ producer
        int64_t issued = 0;
        const int64_t gbase = si.b * p.g_sb + hv * p.g_sh;
        for (int64_t c = 0; c < nchunks; ++c) {
            const int s = static_cast<int>(c % STAGES);
            const uint32_t use = static_cast<uint32_t>(c / STAGES);
            bool go = true;
            if (c >= STAGES && lane == 0) go = mbar_wait(&empty[s], (use - 1) & 1, ctl, 0x10);
            if (p.fault_inject && c == 1) go = false;  // test hook: consumers' waits must expire
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (!go) break;
            const int t0 = static_cast<int>(si.bos + c * kChunk);
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], Cfg::kStageTx);
                const int b = static_cast<int>(si.b);
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubK; ++sub)
                    tma_load_4d(&args.maps.k, smem + s * Cfg::kStageBytes + sub * 8192, &full[s], sub * 64,
                                static_cast<int>(kh), t0, b);
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubK; ++sub)
                    tma_load_4d(&args.maps.w, smem + s * Cfg::kStageBytes + Cfg::kTileKBytes + sub * 8192, &full[s],
                                sub * 64, static_cast<int>(hv), t0, b);
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubV; ++sub)
                    tma_load_4d(&args.maps.u, smem + s * Cfg::kStageBytes + 2 * Cfg::kTileKBytes + sub * Cfg::kUSub,
                                &full[s], v0 + sub * Cfg::kSubCols, static_cast<int>(hv), t0, b);
            }
            // gate inputs of the chunk: 64 fp32 values at any stride, 2 per lane
            if (p.g) {
                const int len = static_cast<int>(si.len - c * kChunk < kChunk ? si.len - c * kChunk : kChunk);
                float* gs = reinterpret_cast<float*>(smem + Cfg::kOffG) + 64 * s;
                if (lane < len) cp_async_4(gs + lane, p.g + gbase + (t0 + lane) * p.g_st);
                if (lane + 32 < len) cp_async_4(gs + lane + 32, p.g + gbase + (t0 + lane + 32) * p.g_st);
            }
            cp_async_arrive_noinc(&full[s]);
            ++issued;
        }
        // Drain: never leave the CTA while a load may still land in its
        // shared memory (bounded, and independent of the abort flag).
        if (lane == 0) {
            const int64_t first = issued > STAGES ? issued - STAGES : 0;
            WaitCtl drain{never_flag, p.status, p.timeout_ns};
            for (int64_t c = first; c < issued; ++c)
                mbar_wait(&full[c % STAGES], static_cast<uint32_t>(c / STAGES) & 1, drain, 0x10);
        }
    } else if (warp >= Cfg::kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer (one per chain)
        // The whole warp runs the loop (descriptors stay warp-uniform); one elected
        // lane issues each MMA and commit, so issue does not stall on a divergent branch.
        auto wait_warp = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, ctl, 0x20) ? 1 : 0) != 0;
        };
        // the chain's columns: D1 at [c N, c N + N), D2 at VT + that, its sub-tiles of S and u_c
        const int csub = chain * (Cfg::kChainCols / Cfg::kSubCols);
        const uint32_t d1 = tmem + static_cast<uint32_t>(chain * Cfg::kChainCols);
        const uint32_t d2 = tmem + VT + static_cast<uint32_t>(chain * Cfg::kChainCols);
        const uint32_t s_addr = sbase + Cfg::kOffS + csub * Cfg::kSSubBytes;
        for (int64_t c = 0; c < nchunks; ++c) {
            const int s = static_cast<int>(c % STAGES);
            if (!wait_warp(&full[s], static_cast<uint32_t>(c / STAGES) & 1)) break;
            // descriptors differ only in the start-address field (bits 0-13, 16-byte units)
            const uint64_t a1 = umma_desc_sw128(wc_addr(s), 16, 1024);
            const uint64_t b1 = umma_desc_mn<Cfg::kSwz>(s_addr, Cfg::kSSubBytes);
            if (!wait_warp(s_ready, static_cast<uint32_t>(c) & 1)) break;
            tc_fence_after();
            if (elect_one_sync()) {
#pragma unroll
                for (int kk = 0; kk < K_ / 16; ++kk)
                    tc_mma_bf16(d1, a1 + static_cast<uint64_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4),
                                b1 + static_cast<uint64_t>((kk * 16 * Cfg::kRowB) >> 4), Cfg::kIdesc1, kk > 0 ? 1u : 0u);
                tc_commit(mma1_done);
            }
            __syncwarp();
            if (!wait_warp(vdec_ready, static_cast<uint32_t>(c) & 1)) break;
            tc_fence_after();
            const uint64_t a2 = umma_desc_sw128(kc_addr(s), 8192, 1024);
            const uint64_t b2 = umma_desc_mn<Cfg::kSwz>(uc_addr(s) + csub * Cfg::kUSub, Cfg::kUSub);
            if (elect_one_sync()) {
                // M = K halves (K = 256): rows 128 m.. of k_c start 2 m sub-tiles in
#pragma unroll
                for (int m = 0; m < Cfg::kM2Halves; ++m)
#pragma unroll
                    for (int tt = 0; tt < 4; ++tt)
                        tc_mma_bf16(d2 + m * VT, a2 + static_cast<uint64_t>((m * 2 * 8192 + tt * 2048) >> 4),
                                    b2 + static_cast<uint64_t>((tt * 16 * Cfg::kRowB) >> 4), Cfg::kIdesc2,
                                    tt > 0 ? 1u : 0u);
                tc_commit(mma2_done);
                tc_commit(&empty[s]);
            }
            __syncwarp();
        }
        // Drain: every MMA this warp issued has completed before the TMEM it writes
        // is released (matters only on an abort path).
        if (elect_one_sync()) tc_commit(mma_drain);
        __syncwarp();
        WaitCtl drain{never_flag, p.status, p.timeout_ns};
        mbar_wait(mma_drain, 0, drain, 0x20);
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;          // TMEM lane quadrant
        const int e = warp >> 2;         // column slice
        const int cbase = e * Cfg::kCW;  // first column (within the V tile) of this warp
        const bool ref = REF;
        uint8_t* s_tile = smem + Cfg::kOffS;
        uint8_t* vout = smem + Cfg::kOffVout;
        const int ta = 16 * q + (lane >> 2);  // epi1 token rows ta, ta+8
        const int tb = ta + 8;
        const int pc = 2 * (lane & 3);        // column pair offset inside an 8-column group

        // State rows owned by this thread (epi2 fragment):
        //   K=256: row 128e+32q+lane, columns [0, VT)
        //   K=128: row 32q+lane, columns cbase + [0, CW)
        //   K=64 : rows 16q+lane/4 (+8), columns cbase + 8j + pc + {0,1}
        // Rows at or beyond the caller's K (K < the tile's K_: k_c and w_c arrive
        // zero-filled past K) stay zero and are never stored; so are columns at or
        // beyond V in a partial V tile.
        constexpr int kNState = (K_ >= 128) ? Cfg::kE2Cols : Cfg::kCW / 2;
        const int e2_row = (K_ == 256 ? 128 * e : 0) + 32 * q + lane;  // K >= 128
        const int e2_c0 = (K_ == 256) ? 0 : cbase;
        const int kdim = static_cast<int>(p.K);
        const int64_t vdim = p.V;
        StateRegs<REF, kNState> st;
        auto st_row_col = [&](int i, int& row, int& col) {
            if constexpr (K_ >= 128) {
                row = e2_row;
                col = e2_c0 + i;
            } else {
                // i = 4*j8 + 2*half + bit: j8 = 8-column group, half selects row +8
                const int j8 = i >> 2, half = (i >> 1) & 1, bit = i & 1;
                row = 16 * q + (lane >> 2) + 8 * half;
                col = cbase + 8 * j8 + pc + bit;
            }
        };

        // ---- initial state
        // K=128: this thread's kCW state values are one contiguous run of a row
        // when V is the unit-stride dimension; 16-byte loads then take a quarter
        // (fp32) or an eighth (bf16) of the L1 wavefronts of scalar loads, whose
        // 32 lanes each touch a different row.  Built for the fp32-state 128-column
        // and single-chain 32-column kernels (B=2 T=4096 H=16: 0.093-0.095 ->
        // 0.090-0.092 ms): in the 64-column and reference-arithmetic kernels the extra
        // code slowed the chunk loop more than it saved (1.42 -> 1.52 ms on a
        // 1024-chunk chain; 0.52 -> 0.55 ms with the rounding chain).
        constexpr bool kVecState = ((K_ == 128 && (VT == 128 || (VT == 32 && CH == 1))) || K_ == 256) && !REF;
        const size_t h0_esz = p.h0_dtype == kBF16 ? 2 : 4;
        const uint8_t* h0_run = nullptr;
        // a whole run inside the caller's K x V state
        const bool full_run = K_ >= 128 && e2_row < kdim && v0 + e2_c0 + kNState <= vdim;
        if constexpr (kVecState) {
            if (p.h0 && p.h0_sv == 1 && full_run) {
                const int64_t at = si.n * p.h0_sn + hv * p.h0_sh + e2_row * p.h0_sk + v0 + e2_c0;
                h0_run = reinterpret_cast<const uint8_t*>(p.h0) + at * static_cast<int64_t>(h0_esz);
                if (reinterpret_cast<uintptr_t>(h0_run) & 15) h0_run = nullptr;
            }
        }
        bool h0_loaded = false;
        if constexpr (kVecState) {
            if (h0_run) {
                h0_loaded = true;
                if (p.h0_dtype == kBF16) {
#pragma unroll
                    for (int j = 0; j < kNState / 8; ++j) {
                        const uint4 x = reinterpret_cast<const uint4*>(h0_run)[j];
                        const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = unpack_bf16x2(w4[e]);
                            st.set_pair(8 * j + 2 * e, f.x, f.y);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < kNState / 4; ++j) {
                        const float4 x = reinterpret_cast<const float4*>(h0_run)[j];
                        st.set_pair(4 * j, x.x, x.y);
                        st.set_pair(4 * j + 2, x.z, x.w);
                    }
                }
            }
        }
        if (!h0_loaded) {
            // pairs of adjacent columns of one row; the reference arithmetic rounds the
            // initial state to bf16 (packing does)
#pragma unroll
            for (int i = 0; i < kNState; i += 2) {
                int row, col;
                st_row_col(i, row, col);
                float x0 = 0.0f, x1 = 0.0f;
                if (p.h0 && row < kdim) {
                    const int64_t at = si.n * p.h0_sn + hv * p.h0_sh + row * p.h0_sk;
                    if (v0 + col < vdim) x0 = load_io(p.h0, p.h0_dtype, at + (v0 + col) * p.h0_sv);
                    if (v0 + col + 1 < vdim) x1 = load_io(p.h0, p.h0_dtype, at + (v0 + col + 1) * p.h0_sv);
                }
                st.set_pair(i, x0, x1);
            }
        }
        // Reference arithmetic: whether every state value of the warp is finite (the
        // packed epilogue-2 chain needs it); a chunk on the packed chain keeps it so.
        auto state_all_finite = [&]() {
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < kNState; ++i) m = fmax_nan(m, fabsf(st.get(i)));
            return __all_sync(0xffffffffu, m < INFINITY) != 0;
        };
        bool state_ok = REF ? state_all_finite() : true;
        bool state_recheck = false;
        auto write_state_tile = [&]() {
            if constexpr (K_ >= 128) {
                const int row = e2_row;
#pragma unroll
                for (int j = 0; j < Cfg::kE2Cols / 8; ++j) {
                    uint4 v;
                    v.x = st.pair_bits(8 * j + 0);
                    v.y = st.pair_bits(8 * j + 2);
                    v.z = st.pair_bits(8 * j + 4);
                    v.w = st.pair_bits(8 * j + 6);
                    *reinterpret_cast<uint4*>(s_tile + tile_off<Cfg::kSwz>(row, e2_c0 + 8 * j, Cfg::kSSubBytes)) = v;
                }
            } else {
#pragma unroll
                for (int i = 0; i < kNState; i += 2) {
                    int row, col;
                    st_row_col(i, row, col);
                    *reinterpret_cast<uint32_t*>(s_tile + sw128_off(row, col, Cfg::kSSubBytes)) = st.pair_bits(i);
                }
            }
        };
        // h rows this warp stores, and the columns (within the V tile) of its sub-tiles
        const int h_r0 = (K_ >= 128) ? e2_row - lane : Cfg::kHRows * q;
        const int h_c0 = (K_ >= 128) ? e2_c0 : cbase;
        const int h_nc = (K_ >= 128) ? Cfg::kE2Cols : Cfg::kCW;
        auto store_h = [&](int64_t chunk) {
            // this warp's rows of its sub-tiles -> h[b, boh+chunk, hv, rows, cols]; boxes that
            // lie wholly past K or V are skipped, partial ones are clipped by the tensor map
            if (lane == 0) {
#pragma unroll
                for (int sub = 0; sub < Cfg::kSubV; ++sub) {
                    if (sub * Cfg::kSubCols < h_c0 || sub * Cfg::kSubCols >= h_c0 + h_nc) continue;
                    if (h_r0 >= kdim || v0 + sub * Cfg::kSubCols >= vdim) continue;
                    tma_store_5d(&args.maps.h, s_tile + sub * Cfg::kSSubBytes + h_r0 * Cfg::kRowB,
                                 v0 + sub * Cfg::kSubCols, h_r0, static_cast<int>(hv),
                                 static_cast<int>(si.boh + chunk), static_cast<int>(si.b));
                }
                bulk_commit_group();
            }
        };

        constexpr int kPairs = Cfg::kCW / 4;  // (column block, 8-column group, row half)
        // Pack v_new after MMA2 is released (64-column tiles); the 10-warp 128-column
        // configuration packs it with v_decay to stay within its register budget.
        constexpr bool kDeferVnew = VT <= 64;
        const uint32_t vo_base = Cfg::kSplitVout ? static_cast<uint32_t>(e * Cfg::kVoutRegion) : 0u;

        // kSharedH: the warps at even column slices issue the h stores of their sub-tile
        const bool h_issuer = !Cfg::kSharedH || (e & 1) == 0;
        // kSharedH, issuer: wait until the epilogue warps all wrote S_x (phase x of
        // s_ready; it cannot move on before this warp's next arrival), then store h[x];
        // false when the wait gave up
        auto store_h_shared = [&](int64_t x) {
            bool go = true;
            if (lane == 0) go = mbar_wait(s_ready, static_cast<uint32_t>(x) & 1, ctl, 0x40);
            go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            if (go) store_h(x);
            return go;
        };

        bool ok = true;
        write_state_tile();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if constexpr (Cfg::kSharedH) {
            if (lane == 0) mbar_arrive(s_ready);
            if (nchunks > 0 && h_issuer) ok = store_h_shared(0);
        } else {
            if (nchunks > 0) store_h(0);
            if (lane == 0) mbar_arrive(s_ready);
        }

        for (int64_t c = 0; c < nchunks && ok; ++c) {
            const int s = static_cast<int>(c % STAGES);
            const int64_t t0 = si.bos + c * kChunk;
            const int len = static_cast<int>(si.len - c * kChunk < kChunk ? si.len - c * kChunk : kChunk);
            const bool partial_varlen = p.varlen && len < kChunk;

            // ================= epilogue 1 =================
            // The gates and the u loads need only the stage: they run while MMA1 does.
            if (!mbar_wait(&full[s], static_cast<uint32_t>(c / STAGES) & 1, ctl, 0x40)) { ok = false; break; }
            const float* gs = reinterpret_cast<const float*>(smem + Cfg::kOffG) + 64 * s;
            float g_l = 0.f, g_a = 0.f, g_b = 0.f;
            if (p.g) {
                g_l = gs[len - 1];
                g_a = ta < len ? gs[ta] : g_l;
                g_b = tb < len ? gs[tb] : g_l;
            }
            float gate_a, gate_b, alpha;
            if (ref) {
                gate_a = ref_gate(g_l, g_a);
                gate_b = ref_gate(g_l, g_b);
                alpha = ref_alpha(g_l);
            } else if (p.use_g) {
                gate_a = safe_exp(g_l - g_a);
                gate_b = safe_exp(g_l - g_b);
                alpha = expf(g_l);
            } else {
                gate_a = gate_b = alpha = 1.0f;
            }
            uint8_t* ut = smem + s * Cfg::kStageBytes + 2 * Cfg::kTileKBytes;
            // Three passes (all loads, all arithmetic, all stores) so that the
            // shared-memory latencies overlap instead of chaining pair by pair.
            // Swizzled byte offsets of this thread's (row, column pair) elements in
            // the u / v_decay / v_new tiles.
            uint32_t offs[kPairs];
#pragma unroll
            for (int i = 0; i < kPairs; ++i) {
                const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                offs[i] = tile_off<Cfg::kSwz>(half ? tb : ta, cbase + 32 * cb + 8 * j + pc, Cfg::kUSub);
            }
            uint32_t uraw[kPairs], vds[kPairs], vns[kPairs], vos[kPairs];
#pragma unroll
            for (int i = 0; i < kPairs; ++i) uraw[i] = *reinterpret_cast<const uint32_t*>(ut + offs[i]);
            if (!mbar_wait(mma1_done, static_cast<uint32_t>(c) & 1, ctl, 0x40)) { ok = false; break; }
            tc_fence_after();
            // D1 in 32-column blocks (16 registers each), or one 16-column block
            constexpr int kAccBlk = Cfg::kCW >= 32 ? Cfg::kCW / 32 : 1;
            uint32_t acc[kAccBlk][Cfg::kCW >= 32 ? 16 : 8];
#pragma unroll
            for (int cb = 0; cb < kAccBlk; ++cb) {
                if constexpr (Cfg::kCW >= 32)
                    tmem_ld_16x256b_x4(tmem + ((32u * q) << 16) + static_cast<uint32_t>(cbase + 32 * cb), acc[cb]);
                else
                    tmem_ld_16x256b_x2(tmem + ((32u * q) << 16) + static_cast<uint32_t>(cbase), acc[cb]);
            }
            tmem_wait_ld();
            // v_decay only (the MMA2 operand); v_new is packed after MMA2 is released.
            // Reference arithmetic: when every |u| and every |GEMM output| of the warp lies
            // below 16384 (so u - ws stays in the f16 range) and both gates lie in [0, 1]
            // (so v_new * gate cannot grow), the packed f16x2 chain needs no saturation and
            // gives the scalar chain's bits; any other value in the warp (NaN, inf, out of
            // range) sends the warp through the scalar chain.
            bool packed_ref = false;
            if constexpr (REF) {
                float m = 0.0f;
#pragma unroll
                for (int i = 0; i < kPairs; ++i) {
                    const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                    const float2 uu = unpack_bf16x2(uraw[i]);
                    m = fmax_nan(m, fabsf(uu.x));
                    m = fmax_nan(m, fabsf(uu.y));
                    m = fmax_nan(m, fabsf(__uint_as_float(acc[cb][4 * j + 2 * half])));
                    m = fmax_nan(m, fabsf(__uint_as_float(acc[cb][4 * j + 2 * half + 1])));
                }
                packed_ref = __all_sync(0xffffffffu, m < 16384.0f && gate_a <= 1.0f && gate_b <= 1.0f) != 0;
            }
            if (packed_ref) {
                const __half2 ga = __float2half2_rn(gate_a), gb = __float2half2_rn(gate_b);
#pragma unroll
                for (int i = 0; i < kPairs; ++i) {
                    const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                    const float2 uu = unpack_bf16x2(uraw[i]);
                    uint32_t vd;
                    ref_vnew_vdecay_x2_fast(uu.x, uu.y, __uint_as_float(acc[cb][4 * j + 2 * half]),
                                            __uint_as_float(acc[cb][4 * j + 2 * half + 1]), half ? gb : ga, vns[i], vd);
                    vds[i] = (half ? tb : ta) < len ? vd : 0u;
                    if constexpr (!kDeferVnew) {
                        const float2 f = __half22float2(bits_h2(vns[i]));
                        vos[i] = (half ? tb : ta) < len ? pack_bf16x2(f.x, f.y) : 0u;
                    }
                }
            } else {
#pragma unroll
            for (int i = 0; i < kPairs; ++i) {
                const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                const float gt = half ? gate_b : gate_a;
                const float a0 = __uint_as_float(acc[cb][4 * j + 2 * half + 0]);
                const float a1 = __uint_as_float(acc[cb][4 * j + 2 * half + 1]);
                const float2 uu = unpack_bf16x2(uraw[i]);
                float d0, d1;
                if (ref) {
                    const float vn0 = ref_vnew(uu.x, a0), vn1 = ref_vnew(uu.y, a1);
                    // v_new is an fp16 value here: keep it exactly as a half pair
                    __half2 hv = __floats2half2_rn(vn0, vn1);
                    vns[i] = *reinterpret_cast<uint32_t*>(&hv);
                    d0 = ref_vdecay(vn0, gt);
                    d1 = ref_vdecay(vn1, gt);
                } else {
                    d0 = (uu.x - a0) * gt;
                    d1 = (uu.y - a1) * gt;
                }
                vds[i] = (half ? tb : ta) < len ? pack_bf16x2(d0, d1) : 0u;
                if constexpr (!kDeferVnew) {
                    const float2 f = ref ? __half22float2(*reinterpret_cast<const __half2*>(&vns[i]))
                                         : make_float2(uu.x - a0, uu.y - a1);
                    vos[i] = (half ? tb : ta) < len ? pack_bf16x2(f.x, f.y) : 0u;
                }
            }
            }
            // v_decay first: it is all MMA2 waits for.
#pragma unroll
            for (int i = 0; i < kPairs; ++i) *reinterpret_cast<uint32_t*>(ut + offs[i]) = vds[i];
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(vdec_ready);
            // v_new while MMA2 runs.
            const bool v_stored = p.v_new && !partial_varlen;
            if (kDeferVnew && p.v_new) {
#pragma unroll
                for (int i = 0; i < kPairs; ++i) {
                    const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                    float vn0, vn1;
                    if (ref) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&vns[i]));
                        vn0 = f.x;
                        vn1 = f.y;
                    } else {
                        const float2 uu = unpack_bf16x2(uraw[i]);
                        vn0 = uu.x - __uint_as_float(acc[cb][4 * j + 2 * half + 0]);
                        vn1 = uu.y - __uint_as_float(acc[cb][4 * j + 2 * half + 1]);
                    }
                    vos[i] = (half ? tb : ta) < len ? pack_bf16x2(vn0, vn1) : 0u;
                }
            }
            if (partial_varlen && p.v_new) {
#pragma unroll
                for (int i = 0; i < kPairs; ++i) {
                    const int cb = i >> 3, j = (i >> 1) & 3, half = i & 1;
                    const int t = half ? tb : ta;
                    const int col = cbase + 32 * cb + 8 * j + pc;  // even, and V % 8 == 0: col < V covers the pair
                    if (t < len && v0 + col < vdim) {
                        const int64_t vi = si.b * p.v_sb + (t0 + t) * p.v_st + hv * p.v_sh + v0 + col;
                        *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(p.v_new) + vi) = vos[i];
                    }
                }
            } else if (v_stored) {
                // staging free: the store of chunk c-1 is read (only h[c]'s may be pending;
                // a warp that stores no h has nothing newer than that store)
                if (lane == 0) {
                    if (h_issuer)
                        bulk_wait_group_read1();
                    else
                        bulk_wait_group_read0();
                }
                __syncwarp();
                if constexpr (Cfg::kSplitVout) {
#pragma unroll
                    for (int i = 0; i < kPairs; ++i) {
                        const int j = (i >> 1) & 3, half = i & 1;
                        *reinterpret_cast<uint32_t*>(vout + vo_base + tile_off<64>(half ? tb : ta, 8 * j + pc, 0)) =
                            vos[i];
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < kPairs; ++i) *reinterpret_cast<uint32_t*>(vout + offs[i]) = vos[i];
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (Cfg::kSplitVout) {
                        if (v0 + cbase < vdim)
                            tma_store_4d(&args.maps.v, vout + vo_base + 16 * q * 64, v0 + cbase, static_cast<int>(hv),
                                         static_cast<int>(t0 + 16 * q), static_cast<int>(si.b));
                    } else {
#pragma unroll
                        for (int sub = 0; sub < Cfg::kSubV; ++sub) {
                            if (sub * Cfg::kSubCols < cbase || sub * Cfg::kSubCols >= cbase + Cfg::kCW) continue;
                            if (v0 + sub * Cfg::kSubCols >= vdim) continue;
                            tma_store_4d(&args.maps.v, vout + sub * Cfg::kUSub + 16 * q * Cfg::kRowB,
                                         v0 + sub * Cfg::kSubCols, static_cast<int>(hv), static_cast<int>(t0 + 16 * q),
                                         static_cast<int>(si.b));
                        }
                    }
                    bulk_commit_group();
                }
            }

            // ================= epilogue 2 =================
            if (!mbar_wait(mma2_done, static_cast<uint32_t>(c) & 1, ctl, 0x40)) { ok = false; break; }
            tc_fence_after();
            const bool more = c + 1 < nchunks;
            // S tile free once h[c]'s store is read (chunk c's v_new store may be pending);
            // the wait overlaps the TMEM loads.
            // kSharedH: the issuers then tell the quadrant's other warps (h_read[q], phase c);
            // those wait for it instead.  False when that wait gave up.
            auto wait_s_free = [&]() {
                bool go = true;
                if (lane == 0 && more) {
                    if (h_issuer) {
                        if (v_stored)
                            bulk_wait_group_read1();
                        else
                            bulk_wait_group_read0();
                        if constexpr (Cfg::kSharedH) mbar_arrive(&h_read[q]);
                    } else {
                        go = mbar_wait(&h_read[q], static_cast<uint32_t>(c) & 1, ctl, 0x40);
                    }
                }
                return __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
            };
            bool s_free = true;
            if constexpr (K_ >= 128) {
                // 32-column blocks of two 16-column loads, or one 16-column load
                constexpr int kE2Blk = Cfg::kE2Cols >= 32 ? Cfg::kE2Cols / 32 : 1;
                constexpr int kE2Half = Cfg::kE2Cols >= 32 ? 2 : 1;
                const uint32_t ta2 = tmem + VT * (1 + (K_ == 256 ? e : 0)) + ((32u * q) << 16) + static_cast<uint32_t>(e2_c0);
#pragma unroll
                for (int cb = 0; cb < kE2Blk; ++cb) {
                    uint32_t r[kE2Half][16];
#pragma unroll
                    for (int j = 0; j < kE2Half; ++j) tmem_ld_32x32b_x16(ta2 + 32 * cb + 16 * j, r[j]);
                    if (cb == 0) s_free = wait_s_free();
                    tmem_wait_ld();
                    // Reference arithmetic: the packed chain without saturation applies to a
                    // finite state (tracked across chunks), 0 <= alpha <= 1 and GEMM outputs
                    // below 32768 in magnitude (finite in f16), else the scalar chain.
                    bool packed_ref = false;
                    if constexpr (REF) {
                        float m = 0.0f;
#pragma unroll
                        for (int j = 0; j < kE2Half; ++j)
#pragma unroll
                            for (int i = 0; i < 16; ++i) m = fmax_nan(m, fabsf(__uint_as_float(r[j][i])));
                        packed_ref = __all_sync(0xffffffffu, state_ok && alpha <= 1.0f && m < 32768.0f) != 0;
                    }
                    if (packed_ref) {
                        const __half2 ah = __float2half2_rn(alpha);
#pragma unroll
                        for (int j = 0; j < kE2Half; ++j)
#pragma unroll
                            for (int i = 0; i < 16; i += 2) {
                                const int si2 = 32 * cb + 16 * j + i;
                                const uint32_t up = h2_bits(ref_gemm_to_f16x2(__uint_as_float(r[j][i]),
                                                                              __uint_as_float(r[j][i + 1])));
                                if constexpr (REF) {
                                    st.set_pair_bits(si2, ref_state_bits_fast(st.pair_bits(si2), up, ah));
                                } else {
                                    float s0 = st.get(si2), s1 = st.get(si2 + 1);
                                    ref_state_x2_fast(s0, s1, up, ah);
                                    st.set_pair(si2, s0, s1);
                                }
                            }
                    } else {
                        if constexpr (REF) state_recheck = true;
#pragma unroll
                        for (int j = 0; j < kE2Half; ++j)
#pragma unroll
                            for (int i = 0; i < 16; i += 2) {
                                const int si2 = 32 * cb + 16 * j + i;
                                const float a0 = __uint_as_float(r[j][i]), a1 = __uint_as_float(r[j][i + 1]);
                                const float s0 = st.get(si2), s1 = st.get(si2 + 1);
                                if (ref)
                                    st.set_pair(si2, ref_state(s0, alpha, a0), ref_state(s1, alpha, a1));
                                else
                                    st.set_pair(si2, fmaf(s0, alpha, a0), fmaf(s1, alpha, a1));
                            }
                    }
                }
                if constexpr (REF) {
                    if (state_recheck) {  // warp-uniform: set on the scalar chain only
                        state_ok = state_all_finite();
                        state_recheck = false;
                    }
                }
            } else {
                s_free = wait_s_free();
#pragma unroll
                for (int cb = 0; cb < Cfg::kCW / 32; ++cb) {
                    uint32_t r[16];
                    tmem_ld_16x256b_x4(tmem + VT + ((32u * q) << 16) + static_cast<uint32_t>(cbase + 32 * cb), r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        const float a0 = __uint_as_float(r[i]), a1 = __uint_as_float(r[i + 1]);
                        const float s0 = st.get(16 * cb + i), s1 = st.get(16 * cb + i + 1);
                        if (ref)
                            st.set_pair(16 * cb + i, ref_state(s0, alpha, a0), ref_state(s1, alpha, a1));
                        else
                            st.set_pair(16 * cb + i, fmaf(s0, alpha, a0), fmaf(s1, alpha, a1));
                    }
                }
            }
            if (!s_free) {
                ok = false;
                break;
            }
            if (more) {
                write_state_tile();
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                // MMA1 and the h store both only read the tile
                if constexpr (Cfg::kSharedH) {
                    if (lane == 0) mbar_arrive(s_ready);
                    if (h_issuer && !store_h_shared(c + 1)) {
                        ok = false;
                        break;
                    }
                } else {
                    if (lane == 0) mbar_arrive(s_ready);
                    store_h(c + 1);
                }
            } else {
                tc_fence_before();
            }
        }
        // ---- final state (plain stores; once per task; 16-byte stores of a
        // contiguous row run where the layout allows, as for the initial state)
        if (ok && p.final_state) {
            uint8_t* f_run = nullptr;
            if constexpr (kVecState) {
                if (p.f_sv == 1 && full_run) {
                    const int64_t at = si.n * p.f_sn + hv * p.f_sh + e2_row * p.f_sk + v0 + e2_c0;
                    f_run = reinterpret_cast<uint8_t*>(p.final_state) + at * (p.f_dtype == kBF16 ? 2 : 4);
                    if (reinterpret_cast<uintptr_t>(f_run) & 15) f_run = nullptr;
                }
            }
            if (f_run && p.f_dtype == kBF16) {
#pragma unroll
                for (int j = 0; j < kNState / 8; ++j)
                    reinterpret_cast<uint4*>(f_run)[j] =
                        make_uint4(st.pair_bits(8 * j), st.pair_bits(8 * j + 2), st.pair_bits(8 * j + 4),
                                   st.pair_bits(8 * j + 6));
            } else if (f_run) {
#pragma unroll
                for (int j = 0; j < kNState / 4; ++j)
                    reinterpret_cast<float4*>(f_run)[j] =
                        make_float4(st.get(4 * j), st.get(4 * j + 1), st.get(4 * j + 2), st.get(4 * j + 3));
            } else {
#pragma unroll
                for (int i = 0; i < kNState; ++i) {
                    int row, col;
                    st_row_col(i, row, col);
                    if (row < kdim && v0 + col < vdim)
                        store_io(p.final_state, p.f_dtype,
                                 si.n * p.f_sn + hv * p.f_sh + row * p.f_sk + (v0 + col) * p.f_sv, st.get(i));
                }
            }
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
