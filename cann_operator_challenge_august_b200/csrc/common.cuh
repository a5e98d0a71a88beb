// Shared definitions of the ChunkGatedDeltaRuleFwdH kernels: the launch
// parameter block and the element-wise arithmetic of the two numerics modes.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace cgdr {

constexpr int kChunk = 64;  // BT, fixed by the op (def.cpp:72-74)

enum IoType : int32_t { kBF16 = 1, kF32 = 2 };

// Everything a kernel needs, by value.  Strides are in elements; the
// innermost dimension of every tensor is contiguous.  "t" strides address
// tokens (global, packed for varlen), "h" strides address heads.
struct FwdHParams {
    const void* k;
    const void* w;
    const void* u;
    const float* g;
    const void* h0;
    const int64_t* cu_seqlens;     // varlen only
    const int64_t* chunk_offsets;  // caller-supplied (optional, varlen)
    void* h;
    void* v_new;                   // nullptr: save_new_value = False
    void* final_state;             // nullptr: not stored
    int* status;                   // device status word (workspace)
    const int32_t* seq_chunk_base; // workspace: chunk offset of each sequence (varlen)
    const int32_t* seq_order;      // workspace: sequences longest first (varlen)

    int64_t B, T, HK, H, K, V, N, NT;
    int64_t k_sb, k_st, k_sh;
    int64_t w_sb, w_st, w_sh;
    int64_t u_sb, u_st, u_sh;
    int64_t g_sb, g_st, g_sh;
    int64_t v_sb, v_st, v_sh;
    int64_t h_sb, h_sc, h_sh, h_sk;
    int64_t h0_sn, h0_sh, h0_sk, h0_sv;  // h0_sv: 1, or K for a [.., V, K] (transposed) state
    int64_t f_sn, f_sh, f_sk, f_sv;

    int32_t io_dtype;     // IoType of k, w, u, h, v_new
    int32_t h0_dtype;     // IoType of initial_state
    int32_t f_dtype;      // IoType of final_state
    int32_t numerics;     // 0 reference, 1 fp32 state
    int32_t use_g;
    int32_t varlen;
    int32_t v_tile;
    int32_t n_vtiles;
    int32_t fault_inject;
    int32_t pad_;
    uint64_t timeout_ns;
};

// Sequence geometry of one task.
struct SeqInfo {
    int64_t b;      // batch row of k/w/u/g/v/h
    int64_t bos;    // first token (within the batch row)
    int64_t len;    // tokens
    int64_t boh;    // chunk index of the sequence's first chunk in h
    int64_t n;      // sequence index (initial/final state row)
};

__device__ __forceinline__ SeqInfo seq_info(const FwdHParams& p, int64_t n)
{
    SeqInfo s;
    s.n = n;
    if (p.varlen) {
        s.b = 0;
        s.bos = p.cu_seqlens[n];
        s.len = p.cu_seqlens[n + 1] - s.bos;
        s.boh = p.chunk_offsets ? p.chunk_offsets[n] : p.seq_chunk_base[n];
    } else {
        s.b = n;
        s.bos = 0;
        s.len = p.T;
        s.boh = 0;
    }
    return s;
}

// ---- scalar arithmetic of the reference rounding chain --------------------------
// generate_golden.py:287-292 (cast_to_float16) and :414-441 (chunk update).
// The __f*_rn intrinsics keep every product and sum separately rounded (the
// compiler may not contract them into an FMA that the reference never does).

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) { return __uint_as_float(b16 << 16); }

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// cast_to_float16: round to fp16; finite values beyond the fp16 range
// saturate to +-65504 while inf and NaN pass through.
__device__ __forceinline__ float cast_f16(float x)
{
    const float c = fabsf(x) < INFINITY ? fminf(fmaxf(x, -65504.0f), 65504.0f) : x;
    return round_f16(c);
}

__device__ __forceinline__ float nan_to_zero(float x) { return x != x ? 0.0f : x; }

// ws = nan_to_num(bf16(acc).to(fp16)): the bf16 GEMM output converted to fp16.
__device__ __forceinline__ float ref_gemm_to_f16(float acc) { return nan_to_zero(round_f16(round_bf16(acc))); }

// v_new (fp16 value) from u (bf16 value) and the MMA1 accumulator.
__device__ __forceinline__ float ref_vnew(float u, float acc)
{
    return cast_f16(__fsub_rn(cast_f16(u), ref_gemm_to_f16(acc)));
}

// v_decay operand of MMA2: bf16(fp16(v_new * gate)).
__device__ __forceinline__ float ref_vdecay(float vnew, float gate_f16)
{
    return round_bf16(cast_f16(__fmul_rn(vnew, gate_f16)));
}

// New bf16 state from the old bf16 state, alpha = fp16(exp(fp16(g_last))) and
// the MMA2 accumulator: bf16(bf16(fp16(fp16(S) * alpha)) + bf16(fp16(bf16(acc)))).
__device__ __forceinline__ float ref_state(float s, float alpha_f16, float acc)
{
    const float hd = cast_f16(__fmul_rn(cast_f16(s), alpha_f16));
    const float up = ref_gemm_to_f16(acc);
    return round_bf16(__fadd_rn(round_bf16(hd), round_bf16(up)));
}

// gate = fp16(exp(g_last - g)) (reference), alpha = fp16(exp(fp16(g_last))).
__device__ __forceinline__ float ref_gate(float g_last, float g) { return cast_f16(expf(g_last - g)); }
__device__ __forceinline__ float ref_alpha(float g_last) { return round_f16(expf(cast_f16(g_last))); }

// Triton's safe_exp (docs/problem.txt:272-274).
__device__ __forceinline__ float safe_exp(float x) { return expf(x <= 0.0f ? x : -INFINITY); }

__device__ __forceinline__ float load_io(const void* base, int32_t dt, int64_t i)
{
    if (dt == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
    return reinterpret_cast<const float*>(base)[i];
}

__device__ __forceinline__ void store_io(void* base, int32_t dt, int64_t i, float v)
{
    if (dt == kBF16)
        reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float*>(base)[i] = v;
}

}  // namespace cgdr

namespace cgdr {

// ---- the reference rounding chain, two elements at a time ---------------------------
// Packed f16x2 / bf16x2 arithmetic gives the same bits as the scalar chain above
// for finite operands: an f16 product of two f16 values is exact in fp32, and a
// single f16 (resp. bf16) rounding of a sum equals fp32-then-f16 (resp. bf16)
// rounding because fp32 carries at least 2p+2 bits.  Infinite or NaN operands
// are left to the scalar functions (callers test ref_pair_is_finite first and
// take the scalar path for the whole warp when any lane is not).

__device__ __forceinline__ uint32_t h2_bits(__half2 x) { return *reinterpret_cast<uint32_t*>(&x); }
__device__ __forceinline__ __half2 bits_h2(uint32_t x) { return *reinterpret_cast<__half2*>(&x); }

// fp32 pair -> f16 pair, round to nearest, finite overflow saturating to +-65504
// (cast_to_float16 for finite inputs).
__device__ __forceinline__ uint32_t f16x2_satfinite(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ __half2 h2_saturate(__half2 x)
{
    return __hmax2(__hmin2(x, __float2half2_rn(65504.0f)), __float2half2_rn(-65504.0f));
}

// bf16 GEMM output of an fp32 accumulator pair, converted to f16 (the GEMM-to-f16
// step of the chain, overflow to inf as torch's .to(float16)).
__device__ __forceinline__ __half2 ref_gemm_to_f16x2(float a0, float a1)
{
    const __nv_bfloat162 b = __floats2bfloat162_rn(a0, a1);
    return __floats2half2_rn(__low2float(b), __high2float(b));
}

__device__ __forceinline__ uint32_t bf16x2_of_h2(__half2 x)
{
    const float2 f = __half22float2(x);
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    return *reinterpret_cast<const uint32_t*>(&b);
}

// Epilogue 1 of the reference chain on a pair: v_new (f16 bits) and v_decay (bf16
// bits) from u (bf16 values), the MMA1 accumulator and the f16 gate.  Requires
// |u|, |acc| < 65000 and a finite gate.
__device__ __forceinline__ void ref_vnew_vdecay_x2(float u0, float u1, float a0, float a1, __half2 gate,
                                                   uint32_t& vn_bits, uint32_t& vd_bits)
{
    const __half2 ws = ref_gemm_to_f16x2(a0, a1);
    const __half2 uh = __floats2half2_rn(u0, u1);
    const __half2 vn = h2_saturate(__hsub2_rn(uh, ws));
    const __half2 vd = h2_saturate(__hmul2_rn(vn, gate));
    vn_bits = h2_bits(vn);
    vd_bits = bf16x2_of_h2(vd);
}

// Epilogue 2 of the reference chain on a pair: the new bf16 state from the old
// one, the f16 alpha and the MMA2 accumulator.  Requires finite state, alpha and
// accumulator (an infinite update is exact too, but NaN needs the scalar path).
__device__ __forceinline__ void ref_state_x2(float& s0, float& s1, float a0, float a1, __half2 alpha)
{
    const __half2 sh = bits_h2(f16x2_satfinite(s0, s1));
    const __half2 hd = h2_saturate(__hmul2_rn(sh, alpha));
    const __half2 up = ref_gemm_to_f16x2(a0, a1);
    const uint32_t hb = bf16x2_of_h2(hd), ub = bf16x2_of_h2(up);
    const __nv_bfloat162 sum =
        __hadd2_rn(*reinterpret_cast<const __nv_bfloat162*>(&hb), *reinterpret_cast<const __nv_bfloat162*>(&ub));
    s0 = __low2float(sum);
    s1 = __high2float(sum);
}

// Epilogue 1 of the reference chain on a pair without saturations: exact when
// |u|, |acc| < 16384 (so u - ws stays in the f16 range) and 0 <= gate <= 1 (so
// v_new * gate cannot grow); callers check both for the whole warp first.
__device__ __forceinline__ void ref_vnew_vdecay_x2_fast(float u0, float u1, float a0, float a1, __half2 gate,
                                                        uint32_t& vn_bits, uint32_t& vd_bits)
{
    const __half2 vn = __hsub2_rn(__floats2half2_rn(u0, u1), ref_gemm_to_f16x2(a0, a1));
    vn_bits = h2_bits(vn);
    vd_bits = bf16x2_of_h2(__hmul2_rn(vn, gate));
}

// Epilogue 2 of the reference chain on a pair whose update is already in f16 (bits
// `up`, finite), for a finite state and 0 <= alpha <= 1: the decayed state
// fp16(fp16(S) * alpha) then stays within the f16 range, so it needs no saturation.
__device__ __forceinline__ void ref_state_x2_fast(float& s0, float& s1, uint32_t up, __half2 alpha)
{
    const __half2 sh = bits_h2(f16x2_satfinite(s0, s1));
    const __half2 hd = __hmul2_rn(sh, alpha);
    const uint32_t hb = bf16x2_of_h2(hd), ub = bf16x2_of_h2(bits_h2(up));
    const __nv_bfloat162 sum =
        __hadd2_rn(*reinterpret_cast<const __nv_bfloat162*>(&hb), *reinterpret_cast<const __nv_bfloat162*>(&ub));
    s0 = __low2float(sum);
    s1 = __high2float(sum);
}

// The same on bf16 bits: the state pair in, the new state pair out (no unpacking of
// the bf16x2 sum).
__device__ __forceinline__ uint32_t ref_state_bits_fast(uint32_t s_bits, uint32_t up, __half2 alpha)
{
    const __half2 sh = bits_h2(f16x2_satfinite(__uint_as_float(s_bits << 16), __uint_as_float(s_bits & 0xffff0000u)));
    const __half2 hd = __hmul2_rn(sh, alpha);
    const uint32_t hb = bf16x2_of_h2(hd), ub = bf16x2_of_h2(bits_h2(up));
    const __nv_bfloat162 sum =
        __hadd2_rn(*reinterpret_cast<const __nv_bfloat162*>(&hb), *reinterpret_cast<const __nv_bfloat162*>(&ub));
    return *reinterpret_cast<const uint32_t*>(&sum);
}

// max that propagates NaN (so a NaN operand fails a later `< bound` test)
__device__ __forceinline__ float fmax_nan(float a, float b)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ float max_abs2(float a, float b) { return fmax_nan(fabsf(a), fabsf(b)); }

}  // namespace cgdr
