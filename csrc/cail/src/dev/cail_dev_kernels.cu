// cail_dev_kernels.cu — sm_100a kernels of the NVLink allreduce.
//
// These replace the reference's host-driven exchange + separate reduce
// kernel (src/gpu/cuda/cail_cuda_reduce.cu:44-136 there, launched once per
// PMPI_Sendrecv step): one launch moves the data over NVLink 5 by loading and
// storing peer GPUs' memory directly and applies the MPI operator on the fly.
// The reduction is a bandwidth-bound stream, so the kernels use 16-byte
// vector loads/stores on plain SIMT threads; tensor cores and TMA have no
// role here, and no TMA multicast load exists anywhere in this file.
//
// Cross-GPU synchronisation uses 32-bit epoch flags written with
// st.release.sys into the peers' flag arrays and polled with ld.acquire.sys;
// epochs only grow, so flags never need resetting.  Every poll is bounded by
// %globaltimer: after timeout_ns the kernel records DevStatus and returns,
// leaving the context usable.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../gpu/cail_ops.h"
#include "cail_dev_copier.cuh"
#include "cail_dev_kernels.cuh"

namespace cail {

namespace {

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// 16-byte vector load of (possibly peer) memory, bypassing L1.
__device__ __forceinline__ uint4 ld_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_v4(void *p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// ld_v4 / st_v4 as the copier loop's load/store policy
struct V4 {
    static __device__ __forceinline__ uint4 ld(const void *p) { return ld_v4(p); }
    static __device__ __forceinline__ void st(void *p, uint4 v) { st_v4(p, v); }
};

template <int OP, typename T>
__device__ __forceinline__ uint4 vop(uint4 a, uint4 b) {
    T *pa = reinterpret_cast<T *>(&a);
    const T *pb = reinterpret_cast<const T *>(&b);
#pragma unroll
    for (int i = 0; i < (int)(16 / sizeof(T)); ++i) pa[i] = apply<OP, T>(pa[i], pb[i]);
    return a;
}

// Waits until flag >= epoch (wrap-safe).  Returns false on timeout.
// Acquire polling and per-thread release stores measured faster on B200
// than relaxed polling or stores behind one explicit system fence.
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ bool wait_flag(const uint32_t *flag, uint32_t epoch,
                                          unsigned long long deadline, uint32_t *seen) {
    uint32_t v = ld_acquire_sys(flag);
    while ((int32_t)(v - epoch) < 0) {
        if (globaltimer() > deadline) {
            *seen = v;
            return false;
        }
        v = ld_acquire_sys(flag);
    }
    return true;
}

__device__ void report(DevStatus *st, int rank, int peer, int block, uint32_t epoch, uint32_t seen) {
    if (atomicCAS(&st->code, 0, 1) == 0) {
        st->rank = rank;
        st->waited_on = peer;
        st->block = block;
        st->epoch = epoch;
        st->seen = seen;
        __threadfence_system();
    }
}

// Argument check failure (CAIL_DEVICE_CHECKS): code 2, the check's number in
// waited_on; reported once by CTA 0's thread 0.
__device__ void report_check(DevStatus *st, int rank, int check) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && atomicCAS(&st->code, 0, 2) == 0) {
        st->rank = rank;
        st->waited_on = check;
        st->block = 0;
        st->epoch = 0;
        st->seen = 0;
        __threadfence_system();
    }
}

// ---------------------------------------------------------------- one-shot
__device__ __forceinline__ void push_signal_os(const OneShotArgs &a, int me, int b, uint32_t e) {
    const int t = threadIdx.x;
    if (t < a.P && t != me) st_release_sys(a.flags[t] + kOsFlagBase + me * kMaxBlocks + b, e);
}

// CAIL_DEVICE_CHECKS for the one-shot kernel: 0 when the arguments are
// consistent, else the number of the failed check.
template <typename T>
__device__ int oneshot_check(const OneShotArgs &a) {
    if (a.P < 2 || a.P > kMaxRanks) return 1;
    if (a.G < 1 || a.G > kMaxBlocks || gridDim.x % (unsigned)a.G != 0 || a.rank0 < 0 ||
        a.rank0 + (int)(gridDim.x / (unsigned)a.G) > a.P)
        return 2;
    if (a.piece == 0 || a.piece % 16) return 3;
    if (a.sg < a.G || (size_t)kOsSlots * a.sg * a.P * a.piece > a.area) return 4;
    if (a.bytes % sizeof(T)) return 5;
    for (int q = 0; q < a.P; ++q)
        if (!a.slots[q] || ((uintptr_t)a.slots[q] & 15) || !a.flags[q]) return 7;
    for (int r = a.rank0; r < a.rank0 + (int)(gridDim.x / (unsigned)a.G); ++r) {
        if (!a.src[r] || !a.dst[r] || !a.rounds_done[r]) return 8;
        if (a.vec && ((((uintptr_t)a.src[r]) | ((uintptr_t)a.dst[r])) & 15)) return 8;
        if (((uintptr_t)a.src[r] | (uintptr_t)a.dst[r]) % sizeof(T)) return 8;
    }
    return 0;
}

// n bytes of src into the same slot of every peer's area (not this rank's):
// each vector is loaded once and stored P - 1 times.
template <typename T, bool VEC>
__device__ __forceinline__ void push_to_peers(const OneShotArgs &a, int me, size_t slot, const char *src, size_t n) {
    size_t done = 0;
    if constexpr (VEC) {
        const size_t nv = n / 16;
        for (size_t i = threadIdx.x; i < nv; i += blockDim.x) {
            const uint4 v = ld_v4(src + i * 16);
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q)
                if (q < a.P && q != me) st_v4(a.slots[q] + slot + i * 16, v);
        }
        done = nv * 16;
    }
    for (size_t e = done / sizeof(T) + threadIdx.x; e < n / sizeof(T); e += blockDim.x) {
        const T v = reinterpret_cast<const T *>(src)[e];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
            if (q < a.P && q != me) reinterpret_cast<T *>(a.slots[q] + slot)[e] = v;
    }
}

template <int OP, typename T, bool VEC>
__global__ void __launch_bounds__(512, 2) oneshot_kernel(OneShotArgs a) {
    __shared__ int s_fail;
    if (a.checks) {
        const int bad = oneshot_check<T>(a);
        if (bad) {
            report_check(a.status, a.rank0, bad);
            return;
        }
    }
    const int me = a.rank0 + (int)(blockIdx.x / (unsigned)a.G);
    const int b = (int)(blockIdx.x % (unsigned)a.G);
    const int P = a.P;
    const char *src = a.src[me];
    char *dst = a.dst[me];
    if (threadIdx.x == 0) s_fail = 0;
    const uint32_t base = a.rounds_done[me][b];  // read by every thread before thread 0 updates it
    __syncthreads();
    auto off = [&](uint32_t k) { return ((size_t)k * a.G + b) * a.piece; };
    auto slot_of = [&](uint32_t e, int q) { return (((size_t)(e % kOsSlots) * a.sg + b) * P + q) * a.piece; };
    auto push = [&](uint32_t k) {
        const uint32_t e = base + k + 1;
        const size_t o = off(k);
        push_to_peers<T, VEC>(a, me, slot_of(e, me), src + o, min(a.piece, a.bytes - o));
        __syncthreads();
        push_signal_os(a, me, b, e);
    };
    if (off(0) < a.bytes) push(0);
    uint32_t k = 0;
    for (; off(k) < a.bytes; ++k) {
        const uint32_t e = base + k + 1;
        const size_t o = off(k);
        const size_t n = min(a.piece, a.bytes - o);
        // wait for every peer's piece of round k
        if (threadIdx.x < P && threadIdx.x != me) {
            uint32_t seen = 0;
            const unsigned long long deadline = globaltimer() + a.timeout_ns;
            if (!wait_flag(a.flags[me] + kOsFlagBase + threadIdx.x * kMaxBlocks + b, e, deadline, &seen)) {
                report(a.status, me, threadIdx.x, b, e, seen);
                s_fail = 1;
            }
        }
        __syncthreads();
        if (s_fail) return;
        if (off(k + 1) < a.bytes) push(k + 1);  // look ahead (three rotating slots)
        // fold round k in rank order
        const char *own_in = src + o;
        char *out = dst + o;
        const char *area0 = a.slots[me] + slot_of(e, 0);
        size_t done = 0;
        if constexpr (VEC) {
            const size_t nv = n / 16;
            for (size_t i = threadIdx.x; i < nv; i += blockDim.x) {
                uint4 v[kMaxRanks];
#pragma unroll
                for (int q = 0; q < kMaxRanks; ++q)
                    if (q < P) v[q] = ld_v4((q == me ? own_in : area0 + q * a.piece) + i * 16);
                uint4 acc = v[0];
#pragma unroll
                for (int q = 1; q < kMaxRanks; ++q)
                    if (q < P) acc = vop<OP, T>(acc, v[q]);
                st_v4(out + i * 16, acc);
            }
            done = nv * 16;
        }
        for (size_t el = done / sizeof(T) + threadIdx.x; el < n / sizeof(T); el += blockDim.x) {
            T acc = T();
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q)
                if (q < P) {
                    const T x = reinterpret_cast<const T *>(q == me ? own_in : area0 + q * a.piece)[el];
                    acc = q == 0 ? x : apply<OP, T>(acc, x);
                }
            reinterpret_cast<T *>(out)[el] = acc;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) a.rounds_done[me][b] = base + k;
}

// ---------------------------------------------------------------- two-shot
template <int OP, typename T>
__device__ __forceinline__ void scalar_elem(const TwoShotArgs &a, size_t e) {
    T acc = reinterpret_cast<const T *>(a.src[0])[e];
    for (int q = 1; q < a.P; ++q) acc = apply<OP, T>(acc, reinterpret_cast<const T *>(a.src[q])[e]);
    for (int q = 0; q < a.P; ++q) reinterpret_cast<T *>(a.dst[q])[e] = acc;
}

template <int OP, typename T, bool U2>
__global__ void __launch_bounds__(512) twoshot_kernel(TwoShotArgs a) {
    constexpr int V = 16 / sizeof(T);
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (a.vector_ok) {
        const size_t lo = a.nvec * a.rank / a.P, hi = a.nvec * (a.rank + 1) / a.P;
        const size_t base = a.head * sizeof(T);
        size_t i = lo + tid;
        if constexpr (U2) {
            // two vectors per iteration: 2P independent loads in flight
            for (; i + stride < hi; i += 2 * stride) {
                const size_t o0 = base + i * 16, o1 = o0 + stride * 16;
                uint4 v0[kMaxRanks], v1[kMaxRanks];
#pragma unroll
                for (int q = 0; q < kMaxRanks; ++q)
                    if (q < a.P) {
                        v0[q] = ld_v4(a.src[q] + o0);
                        v1[q] = ld_v4(a.src[q] + o1);
                    }
                uint4 acc0 = v0[0], acc1 = v1[0];
#pragma unroll
                for (int q = 1; q < kMaxRanks; ++q)
                    if (q < a.P) {
                        acc0 = vop<OP, T>(acc0, v0[q]);
                        acc1 = vop<OP, T>(acc1, v1[q]);
                    }
#pragma unroll
                for (int q = 0; q < kMaxRanks; ++q)
                    if (q < a.P) {
                        st_v4(a.dst[q] + o0, acc0);
                        st_v4(a.dst[q] + o1, acc1);
                    }
            }
        }
        for (; i < hi; i += stride) {
            const size_t off = base + i * 16;
            uint4 v[kMaxRanks];
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q)
                if (q < a.P) v[q] = ld_v4(a.src[q] + off);
            uint4 acc = v[0];
#pragma unroll
            for (int q = 1; q < kMaxRanks; ++q)
                if (q < a.P) acc = vop<OP, T>(acc, v[q]);
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q)
                if (q < a.P) st_v4(a.dst[q] + off, acc);
        }
        if (a.rank == 0) {
            const size_t tail0 = a.head + a.nvec * V;
            for (size_t e = tid; e < a.head; e += stride) scalar_elem<OP, T>(a, e);
            for (size_t e = tail0 + tid; e < a.count; e += stride) scalar_elem<OP, T>(a, e);
        }
    } else {
        const size_t lo = a.count * a.rank / a.P, hi = a.count * (a.rank + 1) / a.P;
        for (size_t e = lo + tid; e < hi; e += stride) scalar_elem<OP, T>(a, e);
    }
    // Make the block's peer stores visible system-wide before the kernel
    // retires (the host barrier that follows lets peers read them): one
    // fence per block after the block barrier covers every thread's stores.
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

// ---------------------------------------------------------------- push two-shot
// Bytes of slice q's piece at slice-relative offset ob (0 past the slice end).
__device__ __forceinline__ size_t push_piece_len(const PushArgs &a, int q, size_t ob) {
    const size_t len = a.slice_off[q + 1] - a.slice_off[q];
    return ob < len ? min(a.piece, len - ob) : 0;
}

// n bytes from src to dst.  VEC: both 16-byte aligned, n a multiple of the
// element size; four vectors in flight per thread.  Otherwise element-wise.
template <typename T, bool VEC>
__device__ __forceinline__ void piece_copy(char *dst, const char *src, size_t n) {
    size_t done = 0;
    if constexpr (VEC) {
        constexpr int U = 4;
        const size_t nv = n / 16;
        size_t i = threadIdx.x;
        for (; i + (U - 1) * blockDim.x < nv; i += U * blockDim.x) {
            uint4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = ld_v4(src + (i + u * blockDim.x) * 16);
#pragma unroll
            for (int u = 0; u < U; ++u) st_v4(dst + (i + u * blockDim.x) * 16, v[u]);
        }
        for (; i < nv; i += blockDim.x) st_v4(dst + i * 16, ld_v4(src + i * 16));
        done = nv * 16;
    }
    for (size_t e = done / sizeof(T) + threadIdx.x; e < n / sizeof(T); e += blockDim.x)
        reinterpret_cast<T *>(dst)[e] = reinterpret_cast<const T *>(src)[e];
}

// Waits (threads 0..P-1 but `me`) for flag word `base + t * kMaxBlocks + b`
// of this rank's array to reach e; false (after reporting) on timeout.
__device__ __forceinline__ void push_wait(const PushArgs &a, int me, int b, int base, uint32_t e, int *fail) {
    const int t = threadIdx.x;
    if (t < a.P && t != me) {
        uint32_t seen = 0;
        const unsigned long long deadline = globaltimer() + a.timeout_ns;
        if (!wait_flag(a.flags[me] + base + t * kMaxBlocks + b, e, deadline, &seen)) {
            report(a.status, me, t, b, e, seen);
            *fail = 1;
        }
    }
}

__device__ __forceinline__ void push_signal(const PushArgs &a, int me, int b, int base, uint32_t e) {
    const int t = threadIdx.x;
    if (t < a.P && t != me) st_release_sys(a.flags[t] + base + me * kMaxBlocks + b, e);
}

// CAIL_DEVICE_CHECKS for the push two-shot: 0 when the arguments are
// consistent, else the number of the failed check.
template <typename T>
__device__ int push_check(const PushArgs &a) {
    if (a.P < 2 || a.P > kMaxRanks) return 1;
    if (a.G < 1 || a.G > kMaxBlocks || gridDim.x % (unsigned)a.G != 0 || a.rank0 < 0 ||
        a.rank0 + (int)(gridDim.x / (unsigned)a.G) > a.P)
        return 2;
    if (a.piece == 0 || a.piece % 16) return 3;
    if ((size_t)2 * a.G * a.P * a.piece > a.area) return 4;
    size_t mx = 0;
    if (a.slice_off[0] != 0) return 5;
    for (int q = 0; q < a.P; ++q) {
        if (a.slice_off[q + 1] < a.slice_off[q] || a.slice_off[q] % sizeof(T)) return 5;
        if (a.vec && a.slice_off[q] % 16) return 5;
        mx = max(mx, a.slice_off[q + 1] - a.slice_off[q]);
    }
    if (mx != a.max_slice || a.slice_off[a.P] % sizeof(T)) return 5;
    if (a.rounds < 1 || (size_t)a.rounds * a.G * a.piece < a.max_slice) return 6;
    for (int q = 0; q < a.P; ++q) {
        if (!a.rs[q] || !a.ag[q] || !a.flags[q] || ((uintptr_t)a.rs[q] & 15) || ((uintptr_t)a.ag[q] & 15)) return 7;
    }
    for (int r = a.rank0; r < a.rank0 + (int)(gridDim.x / (unsigned)a.G); ++r) {
        if (!a.src[r] || !a.dst[r]) return 8;
        if (a.vec && ((((uintptr_t)a.src[r]) | ((uintptr_t)a.dst[r])) & 15)) return 8;
        if (((uintptr_t)a.src[r] | (uintptr_t)a.dst[r]) % sizeof(T)) return 8;
    }
    return 0;
}

template <int OP, typename T, bool VEC>
__global__ void __launch_bounds__(512, 2) push_kernel(PushArgs a) {
    __shared__ int s_fail;
    if (a.checks) {
        const int bad = push_check<T>(a);
        if (bad) {
            report_check(a.status, a.rank0, bad);
            return;
        }
    }
    const int me = a.rank0 + (int)(blockIdx.x / (unsigned)a.G);
    const int b = (int)(blockIdx.x % (unsigned)a.G);
    const int P = a.P;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    const char *src = a.src[me];
    char *dst = a.dst[me];
    const size_t slot_stride = a.piece;
    auto round_off = [&](int k) { return ((size_t)k * a.G + b) * a.piece; };
    // 1. reduce-scatter by pushes: the pieces of round k of every other
    //    rank's slice -> that rank's RS slot, then one flag per peer
    auto push_rs = [&](int k) {
        const size_t ob = round_off(k);
        const uint32_t e = a.epoch0 + (uint32_t)k;
        const size_t my_slot = (((e & 1u) * a.G + b) * P + me) * slot_stride;
        for (int q = 0; q < P; ++q) {
            if (q == me) continue;
            const size_t n = push_piece_len(a, q, ob);
            if (n) piece_copy<T, VEC>(a.rs[q] + my_slot, src + a.slice_off[q] + ob, n);
        }
        __syncthreads();
        push_signal(a, me, b, kRsFlagBase, e);
    };
    if (round_off(0) < a.max_slice) push_rs(0);
    for (int k = 0; k < a.rounds; ++k) {
        const size_t ob = round_off(k);
        if (ob >= a.max_slice) break;  // the same on every rank
        const uint32_t e = a.epoch0 + (uint32_t)k;
        const size_t par = e & 1u;
        const size_t my_slot = ((par * a.G + b) * P + me) * slot_stride;
        push_wait(a, me, b, kRsFlagBase, e, &s_fail);
        __syncthreads();
        if (s_fail) return;

        // 2. fold the own slice's piece in rank order; result -> own output
        //    and every peer's AG slot (pointers formed per unrolled source, so
        //    nothing is indexed at run time)
        {
            const size_t n = push_piece_len(a, me, ob);
            const char *own_in = src + a.slice_off[me] + ob;
            char *own_out = dst + a.slice_off[me] + ob;
            const char *rs0 = a.rs[me] + (par * a.G + b) * P * slot_stride;
            size_t done = 0;
            if constexpr (VEC) {
                const size_t nv = n / 16;
                for (size_t i = threadIdx.x; i < nv; i += blockDim.x) {
                    uint4 v[kMaxRanks];
#pragma unroll
                    for (int q = 0; q < kMaxRanks; ++q)
                        if (q < P) v[q] = ld_v4((q == me ? own_in : rs0 + q * slot_stride) + i * 16);
                    uint4 acc = v[0];
#pragma unroll
                    for (int q = 1; q < kMaxRanks; ++q)
                        if (q < P) acc = vop<OP, T>(acc, v[q]);
#pragma unroll
                    for (int q = 0; q < kMaxRanks; ++q)
                        if (q < P) st_v4((q == me ? own_out : a.ag[q] + my_slot) + i * 16, acc);
                }
                done = nv * 16;
            }
            for (size_t el = done / sizeof(T) + threadIdx.x; el < n / sizeof(T); el += blockDim.x) {
                T acc = T();
#pragma unroll
                for (int q = 0; q < kMaxRanks; ++q)
                    if (q < P) {
                        const T x = reinterpret_cast<const T *>(q == me ? own_in : rs0 + q * slot_stride)[el];
                        acc = q == 0 ? x : apply<OP, T>(acc, x);
                    }
#pragma unroll
                for (int q = 0; q < kMaxRanks; ++q)
                    if (q < P) reinterpret_cast<T *>(q == me ? own_out : a.ag[q] + my_slot)[el] = acc;
            }
        }
        __syncthreads();
        push_signal(a, me, b, kAgFlagBase, e);

        // look ahead: round k + 1's reduce-scatter goes out before this
        // round's gather is waited for.  Its RS slots (the parity of round
        // k - 1) are free: each peer raised AG for round k - 1, which this CTA
        // received in the previous iteration, only after it had folded them.
        if (k + 1 < a.rounds && round_off(k + 1) < a.max_slice) push_rs(k + 1);

        push_wait(a, me, b, kAgFlagBase, e, &s_fail);
        __syncthreads();
        if (s_fail) return;

        // 3. all-gather: the peers' reduced pieces -> own output
        for (int q = 0; q < P; ++q) {
            if (q == me) continue;
            const size_t n = push_piece_len(a, q, ob);
            const size_t slot = ((par * a.G + b) * P + q) * slot_stride;
            if (n) piece_copy<T, VEC>(dst + a.slice_off[q] + ob, a.ag[me] + slot, n);
        }
    }
}

// ---------------------------------------------------------------- NVLS
// multimem forms accepted by ptxas for sm_100a (probed): add on u32, u64
// (also serves s32/s64: wrapping addition has the same bits), f32 (also as
// .v4) and f64; min/max on u32, s32, u64, s64.  No PROD, no 8/16-bit
// integers, no floating-point min/max: those pairs stay on the P2P kernels.
template <int OP, int EC> struct Mm { static constexpr bool ok = false; };

// Each supported pair provides V (the value of one multimem unit), ld (the
// reduction of one unit over all GPUs, through the multicast address) and st
// (its broadcast to all GPUs).
#define CAIL_MM_SCALAR(OPC, ECC, PTX, CT, CONS)                                                 \
    template <> struct Mm<OPC, ECC> {                                                           \
        static constexpr bool ok = true;                                                        \
        static constexpr int bytes = sizeof(CT);                                                \
        using V = CT;                                                                           \
        static __device__ __forceinline__ V ld(const char *mc) {                                \
            CT v;                                                                               \
            asm volatile("multimem.ld_reduce.relaxed.sys.global." PTX " %0, [%1];"             \
                         : "=" CONS(v) : "l"(mc) : "memory");                                   \
            return v;                                                                           \
        }                                                                                       \
        static __device__ __forceinline__ void st(char *mc, V v) {                              \
            asm volatile("multimem.st.relaxed.sys.global." PTX_ST_##ECC " [%0], %1;"           \
                         ::"l"(mc), CONS(v) : "memory");                                        \
        }                                                                                       \
    };
#define PTX_ST_CAIL_EC_U32 "u32"
#define PTX_ST_CAIL_EC_I32 "b32"
#define PTX_ST_CAIL_EC_U64 "u64"
#define PTX_ST_CAIL_EC_I64 "b64"
#define PTX_ST_CAIL_EC_F64 "f64"

CAIL_MM_SCALAR(CAIL_SUM, CAIL_EC_U32, "add.u32", unsigned, "r")
CAIL_MM_SCALAR(CAIL_SUM, CAIL_EC_U64, "add.u64", unsigned long long, "l")
CAIL_MM_SCALAR(CAIL_SUM, CAIL_EC_F64, "add.f64", double, "d")
CAIL_MM_SCALAR(CAIL_MAX, CAIL_EC_U32, "max.u32", unsigned, "r")
CAIL_MM_SCALAR(CAIL_MAX, CAIL_EC_I32, "max.s32", unsigned, "r")
CAIL_MM_SCALAR(CAIL_MAX, CAIL_EC_U64, "max.u64", unsigned long long, "l")
CAIL_MM_SCALAR(CAIL_MAX, CAIL_EC_I64, "max.s64", unsigned long long, "l")
CAIL_MM_SCALAR(CAIL_MIN, CAIL_EC_U32, "min.u32", unsigned, "r")
CAIL_MM_SCALAR(CAIL_MIN, CAIL_EC_I32, "min.s32", unsigned, "r")
CAIL_MM_SCALAR(CAIL_MIN, CAIL_EC_U64, "min.u64", unsigned long long, "l")
CAIL_MM_SCALAR(CAIL_MIN, CAIL_EC_I64, "min.s64", unsigned long long, "l")

template <> struct Mm<CAIL_SUM, CAIL_EC_F32> {
    static constexpr bool ok = true;
    static constexpr int bytes = 16;
    using V = float4;
    static __device__ __forceinline__ V ld(const char *mc) {
        V v;
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(mc) : "memory");
        return v;
    }
    static __device__ __forceinline__ void st(char *mc, V v) {
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};"
                     ::"l"(mc), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
    }
};

__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Cross-rank meeting of CTA b for one step, called by thread 0 after a block
// barrier: a system-scope fence orders the CTA's earlier stores (made
// visible to the block by the barrier) before the release of the
// multimem.red that adds 1 to counter `ctr` on every GPU; then it polls this
// GPU's copy of the counter until `target` arrivals.  false on timeout.
__device__ __forceinline__ bool nvls_meet(const NvlsArgs &a, size_t ctr, uint32_t target, int b, int which) {
    __threadfence_system();
    fence_proxy_alias();
    asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(a.mc_ctr + ctr), "r"(1u) : "memory");
    uint32_t seen = 0;
    const unsigned long long deadline = globaltimer() + a.timeout_ns;
    if (!wait_flag(reinterpret_cast<const uint32_t *>(a.uc_ctr + ctr), target, deadline, &seen)) {
        report(a.status, a.rank, -1 - which, b, target, seen);
        return false;
    }
    return true;
}

// CAIL_DEVICE_CHECKS for the NVLS kernel: 0 when the arguments are
// consistent, else the number of the failed check.
template <typename T, int MB>
__device__ int nvls_check(const NvlsArgs &a) {
    if (a.P < 2 || a.P > kMaxRanks || a.rank < 0 || a.rank >= a.P) return 1;
    if (gridDim.x > (unsigned)kMaxBlocks) return 2;
    if (a.unit == 0 || a.unit % 16 || a.unit % MB) return 3;
    if ((size_t)gridDim.x * 2 * a.unit > a.area) return 4;
    if (((uintptr_t)a.uc | (uintptr_t)a.mc) & 15) return 5;
    if (!a.src || !a.dst || !a.mc_ctr || !a.uc_ctr || !a.steps) return 6;
    if (a.bytes % sizeof(T) || ((uintptr_t)a.src | (uintptr_t)a.dst) % sizeof(T)) return 7;
    return 0;
}

// Warp roles of the NVLS kernel (kNvlsCopiers copier threads, see
// cail_dev_copier.cuh); thread kNvlsLeader (the first reducer) meets the
// other ranks.
constexpr int kNvlsReducers = 512 - kNvlsCopiers;
constexpr int kNvlsLeader = kNvlsCopiers;

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"((uint32_t)__cvta_generic_to_shared(bar)) : "memory");
}
// Waits for the phase with the given parity to complete; false when the
// deadline passed or *fail was raised meanwhile.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned long long deadline,
                                          volatile int *fail) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(bar);
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if (*fail || globaltimer() > deadline) return false;
    }
}

// One CTA per staging pair: copier warps move unit k + 1 in and unit k - 1
// out while the reducer warps run unit k through the switch, so the local
// copies overlap the NVLink traffic.  Slot k % 2 holds unit k; the copiers
// refill it (unit k + 2) only after barrier B of unit k, after which no rank
// touches it until barrier A of unit k + 2.  Hand-offs inside the CTA go
// through shared-memory mbarriers: full[s] (all copier threads arrive after
// a copy-in) and done[s] (the leader arrives after barrier B).
template <int OP, int EC>
__global__ void __launch_bounds__(512, 2) nvls_kernel(NvlsArgs a) {
    using T = typename EcType<EC>::T;
    using M = Mm<OP, EC>;
    __shared__ int s_fail;
    __shared__ __align__(8) uint64_t full[2], done[2];
    if (a.checks) {
        const int bad = nvls_check<T, M::bytes>(a);
        if (bad) {
            report_check(a.status, a.rank, bad);
            return;
        }
    }
    const int b = blockIdx.x;
    const int G = gridDim.x;
    const int tid = threadIdx.x;
    const uint32_t base = a.steps[b];  // read by every thread before the leader updates it
    // units of this CTA: b, b + G, ...
    const size_t units = (a.bytes + a.unit - 1) / a.unit;
    const uint32_t K = (uint32_t)((units - b + G - 1) / G);
    if (tid == 0) {
        s_fail = 0;
        mbar_init(&full[0], kNvlsCopiers);
        mbar_init(&full[1], kNvlsCopiers);
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    volatile int *fail = &s_fail;
    auto slot_uc = [&](uint32_t k) { return a.uc + ((size_t)b * 2 + (k & 1)) * a.unit; };
    auto slot_mc = [&](uint32_t k) { return a.mc + ((size_t)b * 2 + (k & 1)) * a.unit; };
    auto unit_off = [&](uint32_t k) { return ((size_t)k * G + b) * a.unit; };
    auto unit_len = [&](uint32_t k) { return min(a.unit, a.bytes - unit_off(k)); };

    if (tid < kNvlsCopiers) {
        for (uint32_t k = 0; k < K + 2; ++k) {
            if (k >= 2) {  // copy-out of unit k - 2 (needs its barrier B)
                const uint32_t j = k - 2;
                if (!mbar_wait(&done[j & 1], (j >> 1) & 1, globaltimer() + 4 * a.timeout_ns, fail)) return;
                fence_proxy_alias();
                copier_copy<T, V4>(a.dst + unit_off(j), slot_uc(j), unit_len(j), tid);
            }
            if (k < K) {  // copy-in of unit k into the slot just emptied
                copier_copy<T, V4>(slot_uc(k), a.src + unit_off(k), unit_len(k), tid);
                mbar_arrive(&full[k & 1]);
            }
        }
        return;
    }

    // reducers (no early exit: every reducer reaches every named barrier)
    const int rt = tid - kNvlsCopiers;
    constexpr int U = 4;  // multimem units in flight per thread
    const size_t ctr_a = (size_t)b * kNvlsCtrStride;
    const size_t ctr_b = ((size_t)kMaxBlocks + b) * kNvlsCtrStride;
    uint32_t k = 0;
    for (; k < K; ++k) {
        const uint32_t target = (base + k + 1) * (uint32_t)a.P;
        if (!mbar_wait(&full[k & 1], (k >> 1) & 1, globaltimer() + 4 * a.timeout_ns, fail)) *fail = 1;
        if (tid == kNvlsLeader && !*fail && !nvls_meet(a, ctr_a, target, b, 0)) *fail = 1;
        asm volatile("bar.sync 1, %0;" ::"n"(kNvlsReducers) : "memory");
        if (*fail) break;
        fence_proxy_alias();
        // this rank's share of the unit through the switch; the last multimem
        // unit may reach past the data into the slot's padding, which is
        // never copied out
        const size_t n = unit_len(k);
        const size_t mu = (n + M::bytes - 1) / M::bytes;
        const size_t lo = mu * a.rank / a.P, hi = mu * (a.rank + 1) / a.P;
        char *mc = slot_mc(k);
        for (size_t u = lo + rt; u < hi; u += U * kNvlsReducers) {
            typename M::V v[U];
#pragma unroll
            for (int q = 0; q < U; ++q)
                if (u + q * kNvlsReducers < hi) v[q] = M::ld(mc + (u + q * kNvlsReducers) * M::bytes);
#pragma unroll
            for (int q = 0; q < U; ++q)
                if (u + q * kNvlsReducers < hi) M::st(mc + (u + q * kNvlsReducers) * M::bytes, v[q]);
        }
        asm volatile("bar.sync 2, %0;" ::"n"(kNvlsReducers) : "memory");
        if (tid == kNvlsLeader) {
            if (!nvls_meet(a, ctr_b, target, b, 1)) *fail = 1;
            mbar_arrive(&done[k & 1]);  // also on failure: the copiers then see the flag
        }
    }
    if (tid == kNvlsLeader && !*fail) a.steps[b] = base + K;
}

// ---------------------------------------------------------------- fold
// dst = src[0] op src[1] op ... op src[P-1], all local memory; 16-byte
// vectors when every pointer is 16-byte aligned, two per iteration.
template <int OP, typename T>
__global__ void __launch_bounds__(512) fold_kernel(FoldArgs a) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    uintptr_t mis = (uintptr_t)a.dst;
    for (int q = 0; q < a.P; ++q) mis |= (uintptr_t)a.src[q];
    const size_t nv = (mis & 15) == 0 ? a.count * sizeof(T) / 16 : 0;
    size_t i = tid;
    for (; i + stride < nv; i += 2 * stride) {
        uint4 v0[kMaxRanks], v1[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
            if (q < a.P) {
                v0[q] = ld_v4(a.src[q] + i * 16);
                v1[q] = ld_v4(a.src[q] + (i + stride) * 16);
            }
        uint4 acc0 = v0[0], acc1 = v1[0];
#pragma unroll
        for (int q = 1; q < kMaxRanks; ++q)
            if (q < a.P) {
                acc0 = vop<OP, T>(acc0, v0[q]);
                acc1 = vop<OP, T>(acc1, v1[q]);
            }
        st_v4(a.dst + i * 16, acc0);
        st_v4(a.dst + (i + stride) * 16, acc1);
    }
    for (; i < nv; i += stride) {
        uint4 v[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
            if (q < a.P) v[q] = ld_v4(a.src[q] + i * 16);
        uint4 acc = v[0];
#pragma unroll
        for (int q = 1; q < kMaxRanks; ++q)
            if (q < a.P) acc = vop<OP, T>(acc, v[q]);
        st_v4(a.dst + i * 16, acc);
    }
    for (size_t e = nv * 16 / sizeof(T) + tid; e < a.count; e += stride) {
        T acc = reinterpret_cast<const T *>(a.src[0])[e];
        for (int q = 1; q < a.P; ++q) acc = apply<OP, T>(acc, reinterpret_cast<const T *>(a.src[q])[e]);
        reinterpret_cast<T *>(a.dst)[e] = acc;
    }
}

// ---------------------------------------------------------------- copy
// One-rank allreduce: dst = src.  Each thread keeps eight 16-byte loads in
// flight before it stores them.  STREAM (messages whose source and
// destination do not both fit in L2): loads bypass L1 (ld.global.nc, no L1
// allocation) and stores are marked evict-first (st.global.cs), which
// measured 0.0237 ms for 64 MiB on B200 against 0.0292 ms for
// cudaMemcpyAsync.  Otherwise plain cached stores: with both buffers in the
// 126 MB L2, evict-first stores only force write-backs that a cached copy
// avoids (16 MiB, blocking call: 16.0 us with streaming hints against
// 13.4-14.6 us for cudaMemcpy).
template <bool STREAM>
__device__ __forceinline__ uint4 ld_v4_copy(const void *p) {
    uint4 v;
    if constexpr (STREAM)
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(p));
    else
        asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(p));
    return v;
}

template <bool STREAM>
__device__ __forceinline__ void st_v4_copy(void *p, uint4 v) {
    if constexpr (STREAM)
        asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
    else
        asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
}

template <bool STREAM>
__global__ void __launch_bounds__(512) copy_kernel(char *dst, const char *src, size_t head, size_t nvec,
                                                   size_t bytes) {
    constexpr int U = 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint4 *s = reinterpret_cast<const uint4 *>(src + head);
    uint4 *d = reinterpret_cast<uint4 *>(dst + head);
    size_t i = tid;
    for (; i + (U - 1) * stride < nvec; i += U * stride) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = ld_v4_copy<STREAM>(s + i + u * stride);
#pragma unroll
        for (int u = 0; u < U; ++u) st_v4_copy<STREAM>(d + i + u * stride, v[u]);
    }
    for (; i < nvec; i += stride) st_v4_copy<STREAM>(d + i, ld_v4_copy<STREAM>(s + i));
    // ragged head and tail (< 16 bytes each)
    if (tid < head) dst[tid] = src[tid];
    const size_t t0 = head + nvec * 16;
    if (t0 + tid < bytes) dst[t0 + tid] = src[t0 + tid];
}

// ---------------------------------------------------------------- local reduce
template <int OP, typename T>
__global__ void __launch_bounds__(256) reduce_local_kernel(const T *__restrict__ in,
                                                           T *__restrict__ io, size_t n,
                                                           size_t head, size_t nvec, int vec) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (!vec) {
        for (size_t e = tid; e < n; e += stride) io[e] = apply<OP, T>(io[e], in[e]);
        return;
    }
    constexpr int V = 16 / sizeof(T);
    const uint4 *vin = reinterpret_cast<const uint4 *>(in + head);
    uint4 *vio = reinterpret_cast<uint4 *>(io + head);
    for (size_t i = tid; i < nvec; i += stride) vio[i] = vop<OP, T>(vio[i], __ldg(vin + i));
    for (size_t e = tid; e < head; e += stride) io[e] = apply<OP, T>(io[e], in[e]);
    for (size_t e = head + nvec * V + tid; e < n; e += stride) io[e] = apply<OP, T>(io[e], in[e]);
}

}  // namespace

// ---------------------------------------------------------------- launchers
// Functors for dispatch_op_class: one instantiation per (op, storage class).
namespace {

struct LaunchOneShot {
    const OneShotArgs &a;
    int ranks;
    bool coop;
    cudaStream_t s;
    cudaError_t err = cudaSuccess;
    template <int OP, int EC> void operator()() {
        using T = typename EcType<EC>::T;
        void *k = a.vec ? (void *)oneshot_kernel<OP, T, true> : (void *)oneshot_kernel<OP, T, false>;
        const dim3 grid((unsigned)(a.G * ranks)), block(512);
        void *args[] = {(void *)&a};
        err = coop ? cudaLaunchCooperativeKernel(k, grid, block, args, 0, s)
                   : cudaLaunchKernel(k, grid, block, args, 0, s);
    }
};

struct LaunchTwoShot {
    const TwoShotArgs &a;
    int b, t;
    cudaStream_t s;
    template <int OP, int EC> void operator()() {
        if (a.unroll2)
            twoshot_kernel<OP, typename EcType<EC>::T, true><<<b, t, 0, s>>>(a);
        else
            twoshot_kernel<OP, typename EcType<EC>::T, false><<<b, t, 0, s>>>(a);
    }
};

struct LaunchPush {
    const PushArgs &a;
    int ranks;
    bool coop;
    cudaStream_t s;
    cudaError_t err = cudaSuccess;
    template <int OP, int EC> void operator()() {
        using T = typename EcType<EC>::T;
        void *k = a.vec ? (void *)push_kernel<OP, T, true> : (void *)push_kernel<OP, T, false>;
        const dim3 grid((unsigned)(a.G * ranks)), block(512);
        void *args[] = {(void *)&a};
        err = coop ? cudaLaunchCooperativeKernel(k, grid, block, args, 0, s)
                   : cudaLaunchKernel(k, grid, block, args, 0, s);
    }
};

struct LaunchFold {
    const FoldArgs &a;
    int b, t;
    cudaStream_t s;
    template <int OP, int EC> void operator()() {
        fold_kernel<OP, typename EcType<EC>::T><<<b, t, 0, s>>>(a);
    }
};

struct QueryNvls {
    int ok = 0;
    template <int OP, int EC> void operator()() { ok = Mm<OP, EC>::ok ? 1 : 0; }
};

struct LaunchNvls {
    const NvlsArgs &a;
    int b;
    cudaStream_t s;
    bool ok = false;
    template <int OP, int EC> void operator()() {
        if constexpr (Mm<OP, EC>::ok) {
            nvls_kernel<OP, EC><<<b, 512, 0, s>>>(a);
            ok = true;
        }
    }
};

struct LaunchReduceLocal {
    const void *in;
    void *io;
    size_t n;
    int sms;
    cudaStream_t s;
    template <int OP, int EC> void operator()() {
        using T = typename EcType<EC>::T;
        constexpr int V = 16 / sizeof(T);
        uintptr_t ai = (uintptr_t)in, ao = (uintptr_t)io;
        int vec = (ai & 15) == (ao & 15);
        size_t head = vec ? ((16 - (ao & 15)) & 15) / sizeof(T) : 0;
        if (head > n) head = n;
        size_t nvec = vec ? (n - head) / V : 0;
        size_t work = vec ? nvec + 1 : n;
        int threads = 256;
        size_t want = (work + threads - 1) / threads;
        int blocks = (int)(want < (size_t)sms * 8 ? want : (size_t)sms * 8);
        if (blocks < 1) blocks = 1;
        reduce_local_kernel<OP, T><<<blocks, threads, 0, s>>>((const T *)in, (T *)io, n, head, nvec,
                                                             vec);
    }
};

}  // namespace

cudaError_t launch_oneshot(int op, int ec, const OneShotArgs &a, int ranks, bool cooperative, cudaStream_t s) {
    LaunchOneShot l{a, ranks, cooperative, s};
    if (!dispatch_op_class(op, ec, l)) return cudaErrorInvalidValue;
    if (l.err != cudaSuccess) return l.err;
    return cudaGetLastError();
}

cudaError_t launch_twoshot(int op, int ec, const TwoShotArgs &a, int blocks, int threads,
                           cudaStream_t s) {
    LaunchTwoShot l{a, blocks, threads, s};
    if (!dispatch_op_class(op, ec, l)) return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_fold(int op, int ec, const FoldArgs &a, int blocks, int threads, cudaStream_t s) {
    LaunchFold l{a, blocks, threads, s};
    if (!dispatch_op_class(op, ec, l)) return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_push(int op, int ec, const PushArgs &a, int ranks, bool cooperative, cudaStream_t s) {
    LaunchPush l{a, ranks, cooperative, s};
    if (!dispatch_op_class(op, ec, l)) return cudaErrorInvalidValue;
    if (l.err != cudaSuccess) return l.err;
    return cudaGetLastError();
}

int push_max_ctas(int ranks, int sm_count) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, push_kernel<CAIL_SUM, float, true>, 512, 0) !=
            cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    if (per_sm > 2) per_sm = 2;
    int g = per_sm * (sm_count > 0 ? sm_count : 148) / (ranks > 0 ? ranks : 1);
    return g < 1 ? 1 : (g > kMaxBlocks ? kMaxBlocks : g);
}

int nvls_supported(int op, int ec) {
    QueryNvls q;
    if (!dispatch_op_class(op, ec, q)) return 0;
    return q.ok;
}

cudaError_t launch_nvls(int op, int ec, const NvlsArgs &a, int blocks, cudaStream_t s) {
    LaunchNvls l{a, blocks, s};
    if (!dispatch_op_class(op, ec, l) || !l.ok) return cudaErrorInvalidValue;
    return cudaGetLastError();
}

int nvls_max_ctas(int sm_count) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, nvls_kernel<CAIL_SUM, CAIL_EC_F32>, 512, 0) !=
            cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    if (per_sm > 2) per_sm = 2;
    const int g = per_sm * (sm_count > 0 ? sm_count : 148);
    return g > kMaxBlocks ? kMaxBlocks : g;
}

cudaError_t launch_copy(char *dst, const char *src, size_t bytes, int sm_count, cudaStream_t s, bool stream) {
    if (bytes == 0) return cudaSuccess;
    if ((((uintptr_t)src ^ (uintptr_t)dst) & 15) != 0) return cudaErrorInvalidValue;
    size_t head = (16 - ((uintptr_t)src & 15)) & 15;
    if (head > bytes) head = bytes;
    const size_t nvec = (bytes - head) / 16;
    // grid: enough CTAs for about four vectors per thread, at most two
    // 512-thread CTAs per SM (the whole GPU from ~9 MiB up)
    const int threads = 512;
    const size_t want = (nvec + 4 * threads - 1) / (4 * threads);
    const size_t cap = (size_t)(sm_count > 0 ? sm_count : 148) * 2;
    const int blocks = (int)(want < 1 ? 1 : (want > cap ? cap : want));
    if (stream)
        copy_kernel<true><<<blocks, threads, 0, s>>>(dst, src, head, nvec, bytes);
    else
        copy_kernel<false><<<blocks, threads, 0, s>>>(dst, src, head, nvec, bytes);
    return cudaGetLastError();
}

cudaError_t launch_reduce_local(int op, int ec, const void *in, void *io, size_t n, int sm_count,
                                cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    LaunchReduceLocal l{in, io, n, sm_count > 0 ? sm_count : 148, s};
    if (!dispatch_op_class(op, ec, l)) return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace cail
