// cail_noalloc.cu — cail_reduce_sources_noalloc(): the one-shot push / fold
// reduction for callers that cannot allocate device memory.
//
// This file has no counterpart in the reference library.  It is a
// single-GPU variant of cail's one-shot kernel (dev/cail_dev_kernels.cu):
// every CTA first pushes its share of each source into that source's slot
// of a scratch area, then folds the slots in source order into the output.
// Here the sources are buffers of the current device and the scratch area
// is a fixed array compiled into the library, so no call allocates memory.
// See include/cail_noalloc.h for the contract and the limits.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "../core/cail_internal.h"
#include "../gpu/cail_ops.h"
#include "cail_noalloc.h"

namespace {

constexpr int kMaxSrc = CAIL_NOALLOC_MAX_SOURCES;
constexpr size_t kSlot = CAIL_NOALLOC_MAX_BYTES;

// The scratch area: one slot per source.  In host code this name is only a
// stand-in for the symbol; its device address comes from
// cudaGetSymbolAddress() (noalloc_scratch_of below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kMaxSrc * kSlot];

struct Args {
    const char *src[kMaxSrc];
    char *dst;
    char *scratch;  // device address of g_noalloc_scratch
    size_t count;
    int nsrc;
};

template <int OP, typename T>
__device__ __forceinline__ uint4 fold16(uint4 a, uint4 b) {
    T *pa = reinterpret_cast<T *>(&a);
    const T *pb = reinterpret_cast<const T *>(&b);
#pragma unroll
    for (int i = 0; i < (int)(16 / sizeof(T)); ++i) pa[i] = cail::apply<OP, T>(pa[i], pb[i]);
    return a;
}

template <int OP, typename T>
__global__ void __launch_bounds__(512) noalloc_kernel(Args a) {
    const size_t bytes = a.count * sizeof(T);
    const size_t n16 = (bytes + 15) / 16;
    const size_t per = (n16 + gridDim.x - 1) / gridDim.x;
    const size_t lo = min((size_t)blockIdx.x * per, n16) * 16;
    const size_t hi = min(min((size_t)(blockIdx.x + 1) * per, n16) * 16, bytes);

    // 1. push: this block's share of every source into the source's slot
    for (int q = 0; q < a.nsrc; ++q) {
        const char *s = a.src[q];
        char *slot = a.scratch + (size_t)q * kSlot;
        if (((uintptr_t)s & 15) == 0) {
            for (size_t i = lo / 16 + threadIdx.x; i < hi / 16; i += blockDim.x)
                *reinterpret_cast<uint4 *>(slot + i * 16) = *reinterpret_cast<const uint4 *>(s + i * 16);
            for (size_t e = (hi / 16) * 16 / sizeof(T) + threadIdx.x; e < hi / sizeof(T); e += blockDim.x)
                reinterpret_cast<T *>(slot)[e] = reinterpret_cast<const T *>(s)[e];
        } else {
            for (size_t e = lo / sizeof(T) + threadIdx.x; e < hi / sizeof(T); e += blockDim.x)
                reinterpret_cast<T *>(slot)[e] = reinterpret_cast<const T *>(s)[e];
        }
    }
    __syncthreads();  // the same block folds what it pushed: no cross-block sync

    // 2. fold the slots in source order
    const bool dst_vec = ((uintptr_t)a.dst & 15) == 0;
    for (size_t i = lo / 16 + threadIdx.x; i < hi / 16; i += blockDim.x) {
        uint4 acc = *reinterpret_cast<const uint4 *>(a.scratch + i * 16);
        for (int q = 1; q < a.nsrc; ++q)
            acc = fold16<OP, T>(acc, *reinterpret_cast<const uint4 *>(a.scratch + (size_t)q * kSlot + i * 16));
        if (dst_vec) {
            *reinterpret_cast<uint4 *>(a.dst + i * 16) = acc;
        } else {
            const T *pa = reinterpret_cast<const T *>(&acc);
            for (int k = 0; k < (int)(16 / sizeof(T)); ++k) reinterpret_cast<T *>(a.dst + i * 16)[k] = pa[k];
        }
    }
    for (size_t e = (hi / 16) * 16 / sizeof(T) + threadIdx.x; e < hi / sizeof(T); e += blockDim.x) {
        T acc = reinterpret_cast<const T *>(a.scratch)[e];
        for (int q = 1; q < a.nsrc; ++q)
            acc = cail::apply<OP, T>(acc, reinterpret_cast<const T *>(a.scratch + (size_t)q * kSlot)[e]);
        reinterpret_cast<T *>(a.dst)[e] = acc;
    }
}

struct Launch {
    const Args &a;
    int blocks;
    cudaStream_t s;
    template <int OP, int EC> void operator()() {
        noalloc_kernel<OP, typename cail::EcType<EC>::T><<<blocks, 512, 0, s>>>(a);
    }
};

constexpr int kMaxDevices = 64;
std::once_flag g_scratch_once[kMaxDevices];
char *g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on device `dev` (the current device),
// looked up once per device: the first call on a device does the set-up,
// with std::call_once so that concurrent first calls from several host
// threads neither race nor repeat it.  nullptr on failure.
char *noalloc_scratch_of(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return nullptr;
    // a failed lookup throws out of call_once, which leaves the flag unset,
    // so a later call tries again
    try {
        std::call_once(g_scratch_once[dev], [dev] {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess) {
                CAIL_ERR("cail_reduce_sources_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                         cudaGetErrorString(e));
                cudaGetLastError();
                throw e;
            }
            g_scratch_ptr[dev] = (char *)p;
        });
    } catch (cudaError_t) {
        return nullptr;
    }
    return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int cail_reduce_sources_noalloc(const void *const *srcs, int nsrc, void *dst, size_t count,
                                           MPI_Datatype datatype, MPI_Op op, cudaStream_t stream) {
    cail_datatype_t dt = cail_mpi_type_to_dtype(datatype);
    cail_op_t o = cail_mpi_op_to_optype(op);
    if (dt == CAIL_INVALID) return MPI_ERR_TYPE;
    if (o == CAIL_OP_INVALID) return MPI_ERR_OP;
    if (!srcs || !dst) return MPI_ERR_ARG;
    const size_t esz = (size_t)cail_type_size(dt);
    // compared as a count first, so that count * esz cannot wrap
    if (nsrc < 1 || nsrc > kMaxSrc || count > kSlot / esz) {
        CAIL_ERR("cail_reduce_sources_noalloc: %d sources of %zu elements of %zu bytes exceed the limit of %d "
                 "sources of %zu bytes each",
                 nsrc, count, esz, kMaxSrc, kSlot);
        return MPI_ERR_COUNT;
    }
    const size_t bytes = count * esz;
    if (count == 0) return MPI_SUCCESS;
    Args a = {};
    for (int q = 0; q < nsrc; ++q) {
        if (!srcs[q]) return MPI_ERR_ARG;
        a.src[q] = (const char *)srcs[q];
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MPI_ERR_OTHER;
    a.scratch = noalloc_scratch_of(dev);
    if (!a.scratch) return MPI_ERR_OTHER;
    a.dst = (char *)dst;
    a.count = count;
    a.nsrc = nsrc;
    // ~2 vectors per thread, at most one block per 16 KiB of data
    size_t want = (bytes + 16383) / 16384;
    int blocks = (int)(want < 1 ? 1 : (want > 64 ? 64 : want));
    Launch l{a, blocks, stream};
    if (!cail::dispatch_op_class((int)o, (int)cail_elem_class(dt), l)) return MPI_ERR_OP;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        CAIL_ERR("cail_reduce_sources_noalloc: launch failed: %s", cudaGetErrorString(e));
        return MPI_ERR_OTHER;
    }
    return MPI_SUCCESS;
}
