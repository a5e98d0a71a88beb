/*
 * cgdr_varlen.h -- variable-length metadata on the device.
 *
 * The reference derives its chunk list on the host
 * (docs/problem.txt:251-270, prepare_chunk_indices / prepare_chunk_offsets,
 * through a .tolist() of the sequence lengths), which synchronises the host
 * with the device.  This entry point computes the same two tables on the
 * device, on the caller's stream:
 *
 *   chunk_indices [capacity, 2] int64: rows (sequence, chunk within the
 *       sequence) in sequence order; rows past the last chunk are (-1, -1),
 *       which the library's kernels skip;
 *   chunk_offsets [N + 1] int64: the cumulative chunk count of each sequence.
 *
 * capacity = ceil(T / chunk_size) + N - 1 always suffices, so callers can
 * size the recurrence's h for it without reading the lengths back.  If
 * cu_seqlens is not non-decreasing from 0, or needs more rows than the
 * capacity, every row is written as padding and chunk_offsets holds the
 * prefix the lengths gave (the kernels then find no chunk to compute).
 */
#ifndef CGDR_VARLEN_H_
#define CGDR_VARLEN_H_

#include "cgdr_fwd_h.h"

#ifdef __cplusplus
extern "C" {
#endif

/* cu_seqlens int64 [N+1] (device), chunk_indices int64 [capacity, 2],
 * chunk_offsets int64 [N+1] (may be NULL); asynchronous on `stream`. */
cgdrStatus cgdrPrepareChunkIndices(const cgdrTensor* cu_seqlens, int64_t chunk_size, const cgdrTensor* chunk_indices,
                                   const cgdrTensor* chunk_offsets, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CGDR_VARLEN_H_ */
