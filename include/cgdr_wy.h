/*
 * cgdr_wy.h -- C ABI of the WY representation of Gated DeltaNet prefill on
 * B200 (sm_100a): the producer of the hidden-state recurrence's w, u and
 * chunk-local cumulative gate.
 *
 * Per sequence, value head and 64-token chunk (rows i, j of the chunk):
 *     g_c = cumsum of g within the chunk
 *     A   = bf16(k k^T)[i, j] * beta_i * exp(g_c,i - g_c,j)    for j < i, else 0
 *     T   = bf16((I + A)^-1)
 *     w   = bf16(T . bf16(beta * exp(g_c) * k))
 *     u   = bf16(T . bf16(beta * v))
 * This is the reference's stage 1
 * (ref/chunk_gated_delta_rule/tests/pytest/chunk_gated_delta_rule_benchmark.py:55-83,
 * where w appears negated as k_cumdecay; NPU kernel
 * ref/chunk_gated_delta_rule/op_kernel/arch22/chunk_gated_delta_rule_stage1.h).
 * The reference has no separate entry point for it: it runs inside
 * aclnnChunkGatedDeltaRule.  The API follows this library's two-phase
 * shape; its outputs are the inputs of cgdrChunkGatedDeltaRuleFwdH*
 * (token-major layout, g_c as its g).
 *
 * Layout (token-major):
 *     k      [B, T, HK, K]  bf16      v, u [B, T, HV, V]  bf16
 *     beta   [B, T, HV]     bf16      g, g_c [B, T, HV]   fp32 (g optional: no gate;
 *                                                         g_c optional output)
 *     w      [B, T, HV, K]  bf16
 * Variable-length batches (B == 1) pass cu_seqlens int64 [N+1] and
 * chunk_indices int64 [NT, 2] (sequence, chunk-in-sequence).
 *
 * Built configurations: K and V in {64, 128}; k and v with strides that are
 * multiples of 16 bytes and 16-byte aligned bases; w and u likewise.
 */
#ifndef CGDR_WY_H_
#define CGDR_WY_H_

#include "cgdr_fwd_h.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cgdrWyExecutor cgdrWyExecutor;

typedef struct {
    int32_t wait_timeout_ms; /* 0 = default (2000 ms) bound on device-side waits */
    int32_t reserved[7];
} cgdrWyOptions;

/* Phase 1: validates and plans.  g, g_cum, cu_seqlens, chunk_indices and
 * options may be NULL. */
cgdrStatus cgdrChunkGatedDeltaRuleWYGetWorkspaceSize(
    const cgdrTensor* k, const cgdrTensor* v, const cgdrTensor* beta, const cgdrTensor* g,
    const cgdrTensor* cu_seqlens, const cgdrTensor* chunk_indices, int64_t chunk_size,
    const cgdrTensor* w, const cgdrTensor* u, const cgdrTensor* g_cum, const cgdrWyOptions* options,
    uint64_t* workspace_size, cgdrWyExecutor** executor);

/* Phase 2: enqueue on `stream`; consumes `executor`.  The first 256 bytes of
 * the workspace hold the device status word (cgdrReadDeviceStatus). */
cgdrStatus cgdrChunkGatedDeltaRuleWY(void* workspace, uint64_t workspace_size, cgdrWyExecutor* executor,
                                     void* stream);

void cgdrDestroyWyExecutor(cgdrWyExecutor* executor);

#ifdef __cplusplus
}
#endif

#endif /* CGDR_WY_H_ */
