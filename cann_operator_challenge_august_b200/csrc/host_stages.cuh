// Internal entry points of the library's ops for the composed operator
// (cgdr_gdr.cu): each enqueues a planned op on `stream` with a caller-owned
// device status word that it does not clear, so that several ops launched in
// sequence share one status word.  Executors stay owned by the caller.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/cgdr_chunk_o.h"
#include "../../include/cgdr_fwd_h.h"
#include "../../include/cgdr_wy.h"

namespace cgdr {
namespace host {

// Bytes of varlen metadata the recurrence needs after its status header.
uint64_t fwd_h_meta_bytes(const cgdrExecutor* ex);
cgdrStatus fwd_h_enqueue(const cgdrExecutor* ex, int* status, uint8_t* meta, cudaStream_t stream);
cgdrStatus chunk_o_enqueue(const cgdrChunkOExecutor* ex, int* status, cudaStream_t stream);
cgdrStatus wy_enqueue(const cgdrWyExecutor* ex, int* status, cudaStream_t stream);
// The recurrence and the chunk output in one kernel (kernel_ho.cuh), for a
// recurrence plan with K = 128, V in {64, 128}, fp32 state, token-major bf16.
// q [B, T, HK, K] and o [B, T, H, V] are bf16 views with a unit inner stride;
// the plan's h and v_new are neither read nor written.
bool fwd_ho_applies(const cgdrExecutor* ex);
cgdrStatus fwd_ho_enqueue(const cgdrExecutor* ex, const cgdrTensor* q, const cgdrTensor* o, float scale, int* status,
                          uint8_t* meta, cudaStream_t stream);

}  // namespace host
}  // namespace cgdr
