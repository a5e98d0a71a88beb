/*
 * cgdr_gdr.h -- C ABI of the chunked Gated DeltaNet forward operator on B200
 * (sm_100a), composed of this library's three kernels: the WY representation
 * (cgdr_wy.h), the hidden-state recurrence (cgdr_fwd_h.h) and the chunk
 * output (cgdr_chunk_o.h).
 *
 * It is the drop-in counterpart of the reference's full operator
 * aclnnChunkGatedDeltaRule (ref/chunk_gated_delta_rule/op_host/op_api/
 * aclnn_chunk_gated_delta_rule.cpp:125-230), same argument order and
 * meaning, aclTensor* -> cgdrTensor*, aclrtStream -> cudaStream_t:
 *
 *   aclnnChunkGatedDeltaRuleGetWorkspaceSize(query, key, value, beta,
 *       initialState, actualSeqLengths, gOptional, scaleValue, out,
 *       finalState, &workspaceSize, &executor)
 *                             -> cgdrChunkGatedDeltaRuleGetWorkspaceSize
 *   aclnnChunkGatedDeltaRule(workspace, workspaceSize, executor, stream)
 *                             -> cgdrChunkGatedDeltaRule
 *
 * Layout (TND, the reference's; tiling.cpp:375-632 checks the same):
 *     query, key   [T, Nk, Dk]   bf16
 *     value, out   [T, Nv, Dv]   bf16
 *     beta         [T, Nv]       bf16
 *     gOptional    [T, Nv]       fp32 per-token log gate (NULL: no gate)
 *     initialState, finalState [B, Nv, Dv, Dk]  bf16 or fp32
 *     actualSeqLengths [B]       int32, summing to T
 * with 0 < Nk, Nv <= 64, Nv % Nk == 0, 0 < Dk, Dv <= 128 and no empty
 * tensor.  The kernels run at head widths 64 and 128; any other Dk or Dv is
 * zero-padded to the next of the two in the workspace (exact: the padded
 * columns stay zero through every product).  query, key, value and out need
 * contiguous last dimensions, and 16-byte multiple strides where their width
 * is 64 or 128.
 *
 * The recurrence runs with an fp32 state (the fla arithmetic); the output
 * passes the reference's own three-party accuracy check against its fp32
 * golden (ref/chunk_gated_delta_rule/tests/assets/impl/compare.py).
 * The workspace holds the intermediate tensors (chunk-local cumulative
 * gate, w, u, v_new, the per-chunk states h) and the varlen metadata that a
 * device kernel derives from actualSeqLengths, so phase 2 needs no host
 * synchronisation.
 */
#ifndef CGDR_GDR_H_
#define CGDR_GDR_H_

#include "cgdr_fwd_h.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cgdrGdrExecutor cgdrGdrExecutor;

/* Phase 1.  scaleValue <= 0 selects Dk ** -0.5.  gOptional may be NULL. */
cgdrStatus cgdrChunkGatedDeltaRuleGetWorkspaceSize(
    const cgdrTensor* query, const cgdrTensor* key, const cgdrTensor* value, const cgdrTensor* beta,
    const cgdrTensor* initialState, const cgdrTensor* actualSeqLengths, const cgdrTensor* gOptional,
    float scaleValue, const cgdrTensor* out, const cgdrTensor* finalState, uint64_t* workspaceSize,
    cgdrGdrExecutor** executor);

/* Phase 2: enqueue on `stream`; consumes `executor`.  The first 256 bytes of
 * the workspace hold the device status word (cgdrReadDeviceStatus): bit 0x2
 * when actualSeqLengths do not sum to T or hold a negative length. */
cgdrStatus cgdrChunkGatedDeltaRule(void* workspace, uint64_t workspaceSize, cgdrGdrExecutor* executor,
                                   void* stream);

void cgdrDestroyGdrExecutor(cgdrGdrExecutor* executor);

#ifdef __cplusplus
}
#endif

#endif /* CGDR_GDR_H_ */
