// cail_dev_copier.cuh — the copier warps' copy loop of the NVLS kernel.
//
// Kept in its own header so that the same source also compiles as plain host
// C++: a CPU test (csrc/ctests/cail_copier_check.cpp) runs it thread by thread
// in adversarial orders and checks that a slot's copy-out and the copy-in
// that refills it never overlap across threads.  The includer defines
// CAIL_COPIER_FN (default: __device__ __forceinline__) and passes the 16-byte
// load/store as a policy class V with static ld(const void *) -> uint4 and
// st(void *, uint4).
#pragma once

#include <stddef.h>
#include <stdint.h>
#include <vector_types.h>

#ifndef CAIL_COPIER_FN
#define CAIL_COPIER_FN __device__ __forceinline__
#endif

namespace cail {

// Warp roles of the NVLS kernel: the first kNvlsCopyWarps warps copy units
// into and out of the CTA's two staging slots, the others run the multimem
// reduction.
constexpr int kNvlsCopyWarps = 4;
constexpr int kNvlsCopiers = kNvlsCopyWarps * 32;

// n bytes with the copier threads (tid in [0, kNvlsCopiers)).  Thread tid
// moves the 16-byte chunks tid, tid + kNvlsCopiers, ... of the unit, the
// partial last chunk included, whatever the alignment of either end and the
// unit's length.  The copy-out of a slot and the copy-in that refills it
// therefore touch every slot byte from the same thread, in program order,
// and need no barrier between them (a thread that wrote a chunk another
// thread had not yet copied out would corrupt that unit's result).  Both
// ends 16-byte aligned: whole chunks as vectors, four in flight per thread;
// otherwise element by element inside the chunk (an element never straddles
// two chunks: the slot and the unit's offset are 16-byte multiples).
template <typename T, class V>
CAIL_COPIER_FN void copier_copy(char *dst, const char *src, size_t n, int tid) {
    const size_t nv = n / 16;
    if ((((uintptr_t)src | (uintptr_t)dst) & 15) == 0) {
        constexpr int U = 4;
        size_t i = tid;
        for (; i + (U - 1) * kNvlsCopiers < nv; i += U * kNvlsCopiers) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = V::ld(src + (i + u * kNvlsCopiers) * 16);
#pragma unroll
            for (int u = 0; u < U; ++u) V::st(dst + (i + u * kNvlsCopiers) * 16, v[u]);
        }
        for (; i < nv; i += kNvlsCopiers) V::st(dst + i * 16, V::ld(src + i * 16));
    } else {
        constexpr int E = 16 / (int)sizeof(T);
        for (size_t i = tid; i < nv; i += kNvlsCopiers) {
            T v[E];
#pragma unroll
            for (int e = 0; e < E; ++e) v[e] = reinterpret_cast<const T *>(src + i * 16)[e];
#pragma unroll
            for (int e = 0; e < E; ++e) reinterpret_cast<T *>(dst + i * 16)[e] = v[e];
        }
    }
    if (nv % kNvlsCopiers == (size_t)tid)  // the partial last chunk (none when n is a multiple of 16)
        for (size_t off = nv * 16; off < n; off += sizeof(T))
            *reinterpret_cast<T *>(dst + off) = *reinterpret_cast<const T *>(src + off);
}

}  // namespace cail
