// Host helpers shared by the library's entry points: the thread-local error
// message, argument checks on cgdrTensor views and bf16 tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <initializer_list>

#include "../../include/cgdr_fwd_h.h"

namespace cgdr {
namespace host {

// Thread-local message returned by cgdrGetLastErrorMessage.
extern thread_local char g_err[512];

// Formats the message into g_err and returns `st`.
cgdrStatus fail(cgdrStatus st, const char* fmt, ...);

inline uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

inline bool present(const cgdrTensor* t) { return t != nullptr && t->data != nullptr; }

inline cgdrStatus check_rank(const cgdrTensor* t, int rank, const char* name)
{
    if (t->ndim != rank) return fail(CGDR_STATUS_BAD_RANK, "%s must have rank %d, got %d", name, rank, t->ndim);
    return CGDR_STATUS_SUCCESS;
}

inline cgdrStatus check_inner_contiguous(const cgdrTensor* t, const char* name)
{
    if (t->shape[t->ndim - 1] > 1 && t->strides[t->ndim - 1] != 1)
        return fail(CGDR_STATUS_BAD_STRIDE, "%s must be contiguous in its last dimension", name);
    for (int i = 0; i < t->ndim; ++i)
        if (t->shape[i] < 0 || t->strides[i] < 0)
            return fail(CGDR_STATUS_BAD_STRIDE, "%s has a negative extent or stride", name);
    return CGDR_STATUS_SUCCESS;
}

inline bool shape_is(const cgdrTensor* t, std::initializer_list<int64_t> s)
{
    if (t->ndim != static_cast<int>(s.size())) return false;
    int i = 0;
    for (int64_t x : s)
        if (t->shape[i++] != x) return false;
    return true;
}

// TMA needs 16-byte aligned bases and 16-byte multiple strides (bf16 elements).
inline bool tma_aligned(const cgdrTensor* t)
{
    if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return false;
    for (int i = 0; i < t->ndim - 1; ++i)
        if ((t->strides[i] * 2) % 16 != 0) return false;
    return true;
}

// A bf16 tensor map with 128-byte swizzle (64- or 32-byte with swizzle_bytes = 64 or 32) over `rank` dims given innermost
// first (sizes in elements, strides in elements for dims 1..rank-1).
cgdrStatus make_map(CUtensorMap* map, void* base, int rank, const int64_t* size, const int64_t* stride,
                    const uint32_t* box, const char* name, int swizzle_bytes = 128);

}  // namespace host
}  // namespace cgdr
