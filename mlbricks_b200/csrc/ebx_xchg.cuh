// ebx_xchg.cuh -- device side of the tensor-parallel exchange.
//
// Every partial travels as one 8-byte word {fp32 bits, epoch} written with a
// single store into each rank's region (NVLink for peers).  A reader polls the
// word itself until its upper half equals the epoch it expects, so the value
// and its readiness arrive together: no fence, no counter and no flag word sit
// between the producer's store and the consumer's load.  Two slots (epoch & 1)
// keep a rank that runs one exchange ahead from overwriting words a slower
// rank has not read yet; it cannot run two ahead, because finishing exchange
// E + 1 needs every rank's partials of E + 1, which each rank produces only
// after its own exchange E is complete.
//
// Slot layout: slot (e & 1) of source rank r starts at word
// ((e & 1) * world + r) * slot_words, with slot_words = max_m * max_n of the
// exchange, and word tok * N + row inside it holds (tok, row) of the current
// call.  The slot stride is fixed by the exchange, not by the call, so calls
// of different M or N on one exchange never overlap: a rank one exchange ahead
// writes only slot (E + 1) & 1 while a slower peer still reads slot E & 1.
//
// The epoch lives in device memory (so CUDA graph replays advance it): every
// CTA reads it after griddepcontrol.wait, and the last CTA of the kernel that
// completes an exchange (the fused decode kernel, or the finish kernel) stores
// epoch + 1.
//
// Two-phase form (larger world x M, where storing every partial into every
// region costs world x M x N words per rank): each output belongs to one owner
// rank (a contiguous block of row groups or rows).  Phase 1 stores a rank's
// partial only into its owner's region (slot e & 1, source = this rank, tag e);
// the owner sums all ranks' words in rank order and stores the sum into every
// other rank's region at source = owner, tagged e | 2^31, where the readers
// poll for it.  A rank receives phase-1 words only for its own block and
// phase-2 words only for the other blocks, so the two phases never share a word;
// traffic per rank falls to about 2 x M x N words, for one more hop of latency.
// The slot argument above still holds: finishing exchange E + 1 needs every
// owner's phase-2 words of E + 1, written after those owners finished E.
#pragma once

#include <stdint.h>

#include "ebx_common.cuh"
#include "ebx_internal.h"

namespace ebx {

constexpr int kXchgTimeout = 0x7102;
constexpr uint64_t kXchgWaitNs = 2000000000ull;  // 2 s per exchange wait

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Epoch of the last completed exchange of this rank.
__device__ __forceinline__ uint32_t xchg_epoch(const XchgArgs& xa) {
    return *reinterpret_cast<volatile const uint32_t*>(xa.peer[xa.rank] + kXchgEpochOff);
}

// Words of source rank `src` for epoch `e` inside a region (slot stride
// xa.slot_words = max_m * max_n of the exchange; the call's [M][N] words fill
// the start of the slot).
__device__ __forceinline__ uint64_t* xchg_words(const XchgArgs& xa, uint8_t* region, uint32_t e,
                                                int src) {
    return reinterpret_cast<uint64_t*>(region + kXchgDataOff) +
           (size_t(e & 1u) * size_t(xa.world) + size_t(src)) * size_t(xa.slot_words);
}

// Store this rank's partial of (tok, row) for epoch e into every rank's region.
__device__ __forceinline__ void xchg_push(const XchgArgs& xa, uint32_t e, int M, int N, int tok,
                                          int row, float v) {
    const uint64_t w = (uint64_t(e) << 32) | uint64_t(__float_as_uint(v));
    const size_t off = size_t(tok) * size_t(N) + size_t(row);
#pragma unroll 1
    for (int q = 0; q < xa.world; ++q)
        st_relaxed_sys_u64(xchg_words(xa, xa.peer[q], e, xa.rank) + off, w);
}

// Sum of all ranks' partials of (tok, row) for epoch e, in rank order 0..world-1
// (the same order on every rank, so every rank holds the same bits).  Polls each
// word until it carries epoch e; false if one did not arrive within the limit.
__device__ __forceinline__ bool xchg_gather(const XchgArgs& xa, uint32_t e, int M, int N, int tok,
                                            int row, float& out) {
    uint8_t* own = xa.peer[xa.rank];
    const size_t off = size_t(tok) * size_t(N) + size_t(row);
    float s = 0.0f;
    uint64_t t0 = 0;
#pragma unroll 1
    for (int r = 0; r < xa.world; ++r) {
        const uint64_t* p = xchg_words(xa, own, e, r) + off;
        uint64_t w = ld_relaxed_sys_u64(p);
        while (uint32_t(w >> 32) != e) {
            const uint64_t now = global_ns();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > kXchgWaitNs) {
                return false;
            }
            __nanosleep(16);
            w = ld_relaxed_sys_u64(p);
        }
        const float v = __uint_as_float(uint32_t(w));
        s = r == 0 ? v : s + v;
    }
    out = s;
    return true;
}

constexpr uint32_t kXchgPhase2 = 0x80000000u;  // tag bit of an owner's reduced word

// Owner rank of row group / row `i` out of `n`: contiguous blocks, one per rank.
__device__ __forceinline__ int xchg_owner(const XchgArgs& xa, int i, int n) {
    return int((int64_t(i) * xa.world) / n);
}

// One word {v, tag} into rank q's region at source `src`, offset `off` (slot e & 1).
__device__ __forceinline__ void xchg_put(const XchgArgs& xa, uint32_t e, int q, int src, size_t off,
                                         float v, uint32_t tag) {
    st_relaxed_sys_u64(xchg_words(xa, xa.peer[q], e, src) + off,
                       (uint64_t(tag) << 32) | uint64_t(__float_as_uint(v)));
}

// Poll this rank's word at source `src`, offset `off` until it carries `tag`.
__device__ __forceinline__ bool xchg_wait(const XchgArgs& xa, uint32_t e, int src, size_t off,
                                          uint32_t tag, float& out) {
    const uint64_t* p = xchg_words(xa, xa.peer[xa.rank], e, src) + off;
    uint64_t w = ld_relaxed_sys_u64(p);
    uint64_t t0 = 0;
    while (uint32_t(w >> 32) != tag) {
        const uint64_t now = global_ns();
        if (t0 == 0) {
            t0 = now;
        } else if (now - t0 > kXchgWaitNs) {
            return false;
        }
        __nanosleep(16);
        w = ld_relaxed_sys_u64(p);
    }
    out = __uint_as_float(uint32_t(w));
    return true;
}

// Two-phase exchange of (tok, row), owner `o`.  Phase 1 (every rank, before any
// wait): this rank's partial to the owner.
__device__ __forceinline__ void xchg_push_owner(const XchgArgs& xa, uint32_t e, int o, int N, int tok,
                                                int row, float v) {
    xchg_put(xa, e, o, xa.rank, size_t(tok) * size_t(N) + size_t(row), v, e);
}

// Phase 2: the owner sums every rank's partial in rank order and stores the sum
// into every other rank's region; the others wait for it.  Every rank ends with
// the same bits.  False if a word did not arrive within the limit.
__device__ __forceinline__ bool xchg_reduce_owner(const XchgArgs& xa, uint32_t e, int o, int M, int N,
                                                  int tok, int row, float& out) {
    const size_t off = size_t(tok) * size_t(N) + size_t(row);
    if (o != xa.rank) return xchg_wait(xa, e, o, off, e | kXchgPhase2, out);
    if (!xchg_gather(xa, e, M, N, tok, row, out)) return false;
#pragma unroll 1
    for (int q = 0; q < xa.world; ++q)
        if (q != xa.rank) xchg_put(xa, e, q, xa.rank, off, out, e | kXchgPhase2);
    return true;
}

// Every thread calls this at the very end of the kernel that completes exchange
// e; the last CTA to arrive stores the new epoch (all CTAs read the old one at
// their start, before arriving).
__device__ __forceinline__ void xchg_advance(const XchgArgs& xa, uint32_t e) {
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t* counter = reinterpret_cast<uint32_t*>(xa.peer[xa.rank] + kXchgCounterOff);
        if (atomicAdd(counter, 1u) + 1u == gridDim.x) {
            atomicExch(counter, 0u);
            *reinterpret_cast<volatile uint32_t*>(xa.peer[xa.rank] + kXchgEpochOff) = e;
        }
    }
}

}  // namespace ebx
