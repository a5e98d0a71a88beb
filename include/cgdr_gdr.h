/*
 * cgdr_gdr.h -- C ABI of the chunked Gated DeltaNet forward operator on B200
 * (sm_100a), composed of this library's kernels: the WY representation
 * (cgdr_wy.h), then either the hidden-state recurrence (cgdr_fwd_h.h)
 * followed by the chunk output (cgdr_chunk_o.h), or one kernel that does
 * both.
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
 * gate, w, u; on the three-kernel path also v_new and the per-chunk states
 * h) and the varlen metadata that a device kernel derives from
 * actualSeqLengths, so phase 2 needs no host synchronisation.
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

/* Which kernels phase 2 runs after the WY kernel:
 *   FUSED          one kernel for the recurrence and the chunk output; the
 *                  per-chunk states h and v_new stay on chip (Dk padded to
 *                  128, i.e. 64 < Dk <= 128);
 *   THREE_KERNELS  the recurrence (h and v_new to the workspace), then the
 *                  chunk output;
 *   AUTO           FUSED where it applies and B * Nv >= 74 (half the SMs of
 *                  a B200 hold one (sequence, head) task each), else
 *                  THREE_KERNELS. */
typedef enum {
    CGDR_GDR_PATH_AUTO = 0,
    CGDR_GDR_PATH_FUSED = 1,
    CGDR_GDR_PATH_THREE_KERNELS = 2
} cgdrGdrPath;

typedef struct {
    int32_t path;         /* cgdrGdrPath */
    int32_t reserved[7];  /* zero */
} cgdrGdrOptions;

/* Phase 1 with options (NULL: all defaults).  CGDR_GDR_PATH_FUSED for a
 * shape it does not cover returns CGDR_STATUS_UNSUPPORTED. */
cgdrStatus cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx(
    const cgdrTensor* query, const cgdrTensor* key, const cgdrTensor* value, const cgdrTensor* beta,
    const cgdrTensor* initialState, const cgdrTensor* actualSeqLengths, const cgdrTensor* gOptional,
    float scaleValue, const cgdrTensor* out, const cgdrTensor* finalState, const cgdrGdrOptions* options,
    uint64_t* workspaceSize, cgdrGdrExecutor** executor);

/* The path a plan takes (CGDR_GDR_PATH_FUSED or CGDR_GDR_PATH_THREE_KERNELS). */
cgdrStatus cgdrGetGdrPath(const cgdrGdrExecutor* executor, int32_t* path);

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
