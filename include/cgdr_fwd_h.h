/*
 * cgdr_fwd_h.h -- C ABI of the B200 (sm_100a) ChunkGatedDeltaRuleFwdH op.
 *
 * The op is the inter-chunk hidden-state recurrence of Gated DeltaNet
 * prefill.  Per (sequence, value head) and per 64-token chunk c:
 *     h[c]   = S                                  (state before the chunk)
 *     v_new  = u_c - w_c . S                      (stored un-gated)
 *     S      = S * exp(g_last) + k_c^T . (v_new * exp(g_last - g_c))
 *     final  = S after the last chunk
 *
 * The interface is the CUDA counterpart of the reference's generated ACLNN
 * two-phase API (the op definition is
 * code/op_host/chunk_gated_delta_rule_fwd_h_def.cpp:12-74 and the call
 * sequence code/examples/test_aclnn_chunk_gated_delta_rule_fwd_h.cpp:297-326):
 *
 *   aclnnChunkGatedDeltaRuleFwdHGetWorkspaceSize(k, w, u, g, initial_state,
 *       cu_seqlens, chunk_indices, chunk_size, h, v, final_state,
 *       &workspaceSize, &executor)                -> cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize
 *   aclnnChunkGatedDeltaRuleFwdH(workspace, workspaceSize, executor, stream)
 *                                                 -> cgdrChunkGatedDeltaRuleFwdH
 *
 * Inputs and outputs are caller-owned device buffers described by
 * cgdrTensor (the aclTensor counterpart: pointer, dtype, shape, strides).
 * The library allocates no device memory: phase 1 reports how many bytes of
 * workspace phase 2 needs, and the caller passes that buffer in.
 * Phase 2 runs asynchronously on the caller's stream.
 *
 * Threading: every entry point is reentrant.  The only mutable state is a
 * thread-local error string (cgdrGetLastErrorMessage).
 */
#ifndef CGDR_FWD_H_H_
#define CGDR_FWD_H_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CGDR_ABI_VERSION 1

/* Return codes.  The reference reports failures as aclnnStatus != 0 after
 * logging (op_host/chunk_gated_delta_rule_fwd_h_infershape.cpp:135-299,
 * op_host/chunk_gated_delta_rule_fwd_h_tiling.cpp:152-261); here each
 * family of failure has its own code and cgdrGetLastErrorMessage() holds
 * the message. */
typedef enum {
    CGDR_STATUS_SUCCESS = 0,
    CGDR_STATUS_NULL_ARGUMENT = 1,   /* a required tensor/pointer is NULL */
    CGDR_STATUS_BAD_RANK = 2,        /* infershape.cpp:149-164 */
    CGDR_STATUS_BAD_DTYPE = 3,       /* infershape.cpp:166-181 */
    CGDR_STATUS_BAD_SHAPE = 4,       /* infershape.cpp:196-288 */
    CGDR_STATUS_BAD_CHUNK_SIZE = 5,  /* infershape.cpp:183-190, tiling.cpp:178-185 */
    CGDR_STATUS_BAD_VARLEN = 6,      /* infershape.cpp:156-159, 244-275 */
    CGDR_STATUS_BAD_STRIDE = 7,      /* innermost dimension not contiguous */
    CGDR_STATUS_UNSUPPORTED = 8,     /* valid op, configuration not built */
    CGDR_STATUS_WORKSPACE_TOO_SMALL = 9,
    CGDR_STATUS_CUDA_ERROR = 10,     /* a CUDA runtime/driver call failed */
    CGDR_STATUS_DEVICE_ERROR = 11,   /* the kernel flagged an error (cgdrReadDeviceStatus) */
    CGDR_STATUS_BAD_EXECUTOR = 12
} cgdrStatus;

typedef enum {
    CGDR_DT_BF16 = 1,
    CGDR_DT_FLOAT32 = 2,
    CGDR_DT_FLOAT16 = 3,
    CGDR_DT_INT64 = 4,
    CGDR_DT_INT32 = 5
} cgdrDataType;

#define CGDR_MAX_DIMS 8

/* A device tensor view (the aclTensor counterpart).  Strides are in
 * elements.  A tensor whose `data` is NULL counts as absent. */
typedef struct {
    void* data;
    int32_t dtype;  /* cgdrDataType */
    int32_t ndim;
    int64_t shape[CGDR_MAX_DIMS];
    int64_t strides[CGDR_MAX_DIMS];
} cgdrTensor;

/* Tensor layouts.
 * HEAD_MAJOR  -- the reference op's layout (infershape.cpp:225-238, 290-297):
 *                k [B,T,HK,K]  w [B,HV,T,K]  u [B,HV,T,V]  g [B,HV,T]
 *                h [B,HV,NT,K,V]  v [B,HV,T,V]  initial/final [N,HV,K,V]
 * TOKEN_MAJOR -- the fla / vLLM layout (docs/problem.txt:434-435, 468-472):
 *                k [B,T,HK,K]  w [B,T,HV,K]  u [B,T,HV,V]  g [B,T,HV]
 *                h [B,NT,HV,K,V]  v [B,T,HV,V]  initial/final [N,HV,K,V] */
typedef enum {
    CGDR_LAYOUT_HEAD_MAJOR = 0,
    CGDR_LAYOUT_TOKEN_MAJOR = 1
} cgdrLayout;

/* Arithmetic of the recurrence.
 * REFERENCE  -- the contest's normative PyTorch reference
 *               (docs/problem.txt:81-167, golden generate_golden.py:350-440):
 *               fp16/bf16 rounding at every point the reference rounds, a
 *               bf16 state between chunks.  bf16 I/O only.
 * FP32_STATE -- the fla / Triton kernel (docs/problem.txt:272-432): fp32
 *               state, bf16 MMA operands for bf16 I/O, safe_exp gating.
 *               The only mode for fp32 I/O. */
typedef enum {
    CGDR_NUMERICS_REFERENCE = 0,
    CGDR_NUMERICS_FP32_STATE = 1
} cgdrNumerics;

/* Extra attributes of the extended phase 1 (zero-initialise for defaults:
 * HEAD_MAJOR layout, REFERENCE numerics, relaxed limits, automatic plan). */
typedef struct {
    int32_t layout;                  /* cgdrLayout */
    int32_t numerics;                /* cgdrNumerics */
    int32_t strict_reference_limits; /* 1: also enforce the reference's
                                        B==1, T<=256K, HK<=32, HV<=128,
                                        32<=K==V<=256, N<=4 limits
                                        (infershape.cpp:196-275) */
    int32_t force_kernel;            /* 0 auto, 1 tensor-core path, 2 general path */
    int32_t v_tile;                  /* 0 auto; else 32 (64 < K <= 128 only), 64 or
                                        128 (64 only for K > 128) */
    int32_t wait_timeout_ms;         /* 0 = default (2000 ms): bound on every
                                        device-side wait before the kernel
                                        gives up and flags DEVICE_ERROR */
    int32_t fault_inject;            /* test hook: 1 makes the load producer
                                        stop after chunk 0 so that the bounded
                                        waits expire; 0 in production */
    int32_t chains;                  /* 0 auto, 1, or 2: the two column halves
                                        of a V tile run as independent chains
                                        in one CTA (64 < K <= 128 with v_tile
                                        32 or 128) */
} cgdrFwdHOptions;

/* Launch plan chosen in phase 1 (the counterpart of the reference's tiling
 * data, op_kernel/chunk_gated_delta_rule_fwd_h_tiling_data.h:11-42). */
typedef struct {
    int64_t batch, total_tokens, key_heads, value_heads, key_dim, value_dim;
    int64_t sequence_count, chunk_count, head_ratio;
    int64_t v_tile, v_tile_count, task_count;
    int32_t has_initial_state, is_varlen, store_final_state, save_new_value;
    int32_t plan_key;        /* has_init | varlen<<1 | store_final<<2, as
                                tiling.cpp:255-259 */
    int32_t kernel;          /* 1 tensor-core (tcgen05) path, 2 general path */
    int32_t grid, block, smem_bytes, stages;
    int32_t numerics, layout;
    uint64_t workspace_bytes;
    int32_t chains;          /* chains per CTA (each v_tile / chains columns);
                                task_count counts chains, grid CTAs */
    int32_t reserved;
} cgdrFwdHPlan;

typedef struct cgdrExecutor cgdrExecutor;

/* Phase 1 (reference argument order).  HEAD_MAJOR layout, REFERENCE
 * numerics, bf16 I/O.  initial_state, cu_seqlens, chunk_indices and
 * final_state may be NULL (or have data == NULL); cu_seqlens and
 * chunk_indices must be both present or both absent.  On success
 * *executor owns the validated plan and must be passed to
 * cgdrChunkGatedDeltaRuleFwdH (which frees it) or cgdrDestroyExecutor. */
cgdrStatus cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize(
    const cgdrTensor* k, const cgdrTensor* w, const cgdrTensor* u, const cgdrTensor* g,
    const cgdrTensor* initial_state, const cgdrTensor* cu_seqlens,
    const cgdrTensor* chunk_indices, int64_t chunk_size,
    const cgdrTensor* h, const cgdrTensor* v, const cgdrTensor* final_state,
    uint64_t* workspace_size, cgdrExecutor** executor);

/* Extended phase 1: as above plus the fla wrapper's knobs
 * (docs/problem.txt:436-447): chunk_offsets (int64 [N+1], optional), v may be
 * NULL (save_new_value=False), g may be NULL in FP32_STATE numerics
 * (USE_G=False), layout/numerics/limits in `options` (NULL = defaults). */
cgdrStatus cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx(
    const cgdrTensor* k, const cgdrTensor* w, const cgdrTensor* u, const cgdrTensor* g,
    const cgdrTensor* initial_state, const cgdrTensor* cu_seqlens,
    const cgdrTensor* chunk_indices, const cgdrTensor* chunk_offsets, int64_t chunk_size,
    const cgdrTensor* h, const cgdrTensor* v, const cgdrTensor* final_state,
    const cgdrFwdHOptions* options, uint64_t* workspace_size, cgdrExecutor** executor);

/* Phase 2: enqueue the op on `stream` (a cudaStream_t; NULL = legacy
 * default stream).  Consumes and frees `executor` whatever the outcome.
 * `workspace` is device memory of at least the size phase 1 returned,
 * 256-byte aligned. */
cgdrStatus cgdrChunkGatedDeltaRuleFwdH(void* workspace, uint64_t workspace_size,
                                       cgdrExecutor* executor, void* stream);

/* Frees an executor that will not be launched. */
void cgdrDestroyExecutor(cgdrExecutor* executor);

/* Copies the plan held by an executor (host-only; no GPU needed). */
cgdrStatus cgdrGetPlan(const cgdrExecutor* executor, cgdrFwdHPlan* plan);

/* Synchronises `stream` and reads the device status word that the last
 * launch using `workspace` left there: 0 = clean; otherwise bit flags
 * (CGDR_DEVICE_* below).  Returns CGDR_STATUS_DEVICE_ERROR when the word
 * is non-zero. */
cgdrStatus cgdrReadDeviceStatus(const void* workspace, uint64_t workspace_size, void* stream,
                                int32_t* device_status);

#define CGDR_DEVICE_WAIT_TIMEOUT 0x1      /* a bounded wait expired */
#define CGDR_DEVICE_BAD_VARLEN 0x2        /* cu_seqlens not increasing / inconsistent */
#define CGDR_DEVICE_TIMEOUT_PRODUCER 0x10 /* which role gave up first */
#define CGDR_DEVICE_TIMEOUT_MMA 0x20
#define CGDR_DEVICE_TIMEOUT_EPILOGUE 0x40

/* Phase 2 without any allocation.  This entry point has no counterpart in
 * the reference (its ACLNN API always returns a workspace size for the
 * caller to allocate).
 *
 * It exists for callers that cannot call cudaMalloc: a plugin or library
 * host that is handed only input/output pointers and a stream while its
 * framework's memory pool owns the device memory (an inference server that
 * reserves almost all HBM for its KV cache up front, for example), or a
 * latency-critical path that must not trigger cudaMalloc's implicit
 * device-wide synchronisation.  Instead of a caller workspace it uses a
 * scratch buffer compiled into this library: a file-scope __device__ array
 * of CGDR_NOALLOC_SCRATCH_BYTES (64 KiB) that every GPU which loads the
 * library holds until the process exits.  Nothing here allocates: no
 * cudaMalloc, no cudaFree, no allocating library routine.
 *
 * - Limit: a plan whose workspace exceeds CGDR_NOALLOC_SCRATCH_BYTES is
 *   rejected with CGDR_STATUS_WORKSPACE_TOO_SMALL before any device work
 *   (fixed-length inputs need 256 bytes; variable-length inputs need about
 *   8 bytes per sequence, so up to roughly 8000 sequences fit).
 * - Device: the buffer of the current device is used; `stream` must belong
 *   to it.  The first call on each device looks up the buffer's address
 *   (cudaGetSymbolAddress) with that device current and keeps it for the life
 *   of the process; make that first call before any stream capture, and do
 *   not reset the device (cudaDeviceReset) between calls, since a reset
 *   invalidates the kept address.  Device ordinals up to 63 are served.
 * - Sharing: every call shares the one buffer, which keeps the last call's
 *   contents; each call clears its status word before its kernels run.
 *   Calls whose work overlaps on the GPU (other streams, other host
 *   threads) race on the buffer: serialise them, e.g. on one stream.
 * - `executor` is consumed whatever the outcome.  If `device_status` is not
 *   NULL the call synchronises `stream` and stores the kernels' status word
 *   there (0 = clean), returning CGDR_STATUS_DEVICE_ERROR when it is not 0;
 *   with NULL the call stays asynchronous. */
#define CGDR_NOALLOC_SCRATCH_BYTES 65536
cgdrStatus cgdrChunkGatedDeltaRuleFwdHNoAlloc(cgdrExecutor* executor, void* stream, int32_t* device_status);

/* Thread-local message describing the last failure on this thread. */
const char* cgdrGetLastErrorMessage(void);

/* ABI version of the loaded library (CGDR_ABI_VERSION). */
int32_t cgdrGetAbiVersion(void);

#ifdef __cplusplus
}
#endif

#endif /* CGDR_FWD_H_H_ */
