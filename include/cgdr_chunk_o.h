/*
 * cgdr_chunk_o.h -- C ABI of the chunk output of Gated DeltaNet prefill on
 * B200 (sm_100a): the consumer of the hidden-state recurrence's h and v_new.
 *
 * Per sequence, value head and 64-token chunk c (rows i, j of the chunk):
 *     o[i] = q'[i] . h[c] + sum_{j <= i} P[i, j] v_new[j]
 *     q'   = bf16(q * scale * exp(g))
 *     P    = bf16(bf16(q k^T) * scale * exp(g_i - g_j))
 * with g the chunk-local cumulative log gate.  This is the inter-chunk term
 * of the reference's stage 2 and its stage 3
 * (ref/chunk_gated_delta_rule/tests/pytest/chunk_gated_delta_rule_benchmark.py:77-79,
 * :129, :145-175; NPU kernel ref/chunk_gated_delta_rule/op_kernel/arch22/
 * chunk_gated_delta_rule_stage3.h:111-180).  The reference has no separate
 * entry point for it: it runs inside aclnnChunkGatedDeltaRule
 * (ref/chunk_gated_delta_rule/op_host/op_api/aclnn_chunk_gated_delta_rule.cpp).
 * The API below follows the same two-phase shape as the rest of this library
 * and the argument set of the fla `chunk_fwd_o` wrapper.
 *
 * Layout (token-major, the fla / vLLM layout):
 *     q, k   [B, T, HK, K]   bf16
 *     v_new  [B, T, HV, V]   bf16
 *     h      [B, NT, HV, K, V] bf16  (state before each chunk)
 *     g      [B, T, HV]      fp32    (optional: no gate when absent)
 *     o      [B, T, HV, V]   bf16
 * Variable-length batches (B == 1) pass cu_seqlens int64 [N+1] and
 * chunk_indices int64 [NT, 2] (sequence, chunk-in-sequence), as the fwd_h op.
 *
 * Built configurations: K in {64, 128}, V a multiple of 64, bf16 I/O, strides
 * that are multiples of 16 bytes (TMA) and 16-byte aligned bases.
 */
#ifndef CGDR_CHUNK_O_H_
#define CGDR_CHUNK_O_H_

#include "cgdr_fwd_h.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cgdrChunkOExecutor cgdrChunkOExecutor;

typedef struct {
    int32_t wait_timeout_ms; /* 0 = default (2000 ms) bound on device-side waits */
    int32_t reserved[7];
} cgdrChunkOOptions;

/* Phase 1: validates and plans.  `scale` <= 0 selects 1/sqrt(K), the
 * reference's default (ref/chunk_gated_delta_rule/tests/assets/impl/golden.py:127-128).
 * g, cu_seqlens, chunk_indices and options may be NULL. */
cgdrStatus cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize(
    const cgdrTensor* q, const cgdrTensor* k, const cgdrTensor* v_new, const cgdrTensor* h, const cgdrTensor* g,
    const cgdrTensor* cu_seqlens, const cgdrTensor* chunk_indices, double scale, int64_t chunk_size,
    const cgdrTensor* o, const cgdrChunkOOptions* options, uint64_t* workspace_size,
    cgdrChunkOExecutor** executor);

/* Phase 2: enqueue on `stream`; consumes `executor`.  The first 256 bytes of
 * the workspace hold the device status word (cgdrReadDeviceStatus). */
cgdrStatus cgdrChunkGatedDeltaRuleFwdO(void* workspace, uint64_t workspace_size, cgdrChunkOExecutor* executor,
                                       void* stream);

void cgdrDestroyChunkOExecutor(cgdrChunkOExecutor* executor);

/* Grid (CTAs) of a planned launch, or -1 for an invalid executor. */
int64_t cgdrChunkOGridSize(const cgdrChunkOExecutor* executor);

#ifdef __cplusplus
}
#endif

#endif /* CGDR_CHUNK_O_H_ */
