/*
 * cail_noalloc.h — a reduction entry point that allocates no memory.
 *
 * This entry point has no counterpart in the reference library; it is an
 * addition of cail-b200.
 *
 * Some callers cannot call cudaMalloc: code that runs inside another
 * allocator's callbacks (a caching allocator cannot re-enter the driver
 * allocator it wraps), code in processes where a framework's caching
 * allocator has already reserved nearly all device memory, and code on
 * latency-critical paths that cannot afford the device-wide synchronisation
 * that cudaMalloc / cudaFree may imply.  For them,
 * cail_reduce_sources_noalloc() folds up to CAIL_NOALLOC_MAX_SOURCES device
 * buffers of the current device into one output with the same push / fold
 * scheme as cail's one-shot allreduce kernel, using a fixed scratch array
 * compiled into the library instead of allocated memory.
 *
 *   out[i] = op(...op(op(src[0][i], src[1][i]), src[2][i])..., src[n-1][i])
 *
 * Limits: at most CAIL_NOALLOC_MAX_SOURCES sources of at most
 * CAIL_NOALLOC_MAX_BYTES bytes each (the scratch array is
 * CAIL_NOALLOC_MAX_SOURCES x CAIL_NOALLOC_MAX_BYTES = 2 MiB, held by every
 * GPU that loads the library until the process exits).  Larger requests are
 * rejected with MPI_ERR_COUNT and an "[cail ERROR]" message.
 *
 * The scratch array is shared by every call on a device and keeps the last
 * call's contents; nothing in it needs to start at zero, because each call
 * writes every scratch byte it later reads.  Calls whose kernels overlap on
 * the GPU (other streams, other host threads) race on that array: serialise
 * them.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  The call is asynchronous with respect to the
 * host: the work is queued on `stream`.
 */
#ifndef CAIL_NOALLOC_H
#define CAIL_NOALLOC_H

#include <cuda_runtime.h>
#include <mpi.h>
#include <stddef.h>

#define CAIL_NOALLOC_MAX_SOURCES 8
#define CAIL_NOALLOC_MAX_BYTES (256u << 10)

#ifdef __cplusplus
extern "C" {
#endif

/* Folds nsrc device buffers of `count` elements of `datatype` (one of the 20
 * datatypes cail supports) with `op` (MPI_SUM, MPI_PROD, MPI_MAX, MPI_MIN) in
 * source order into `dst`, on `stream`.  Returns MPI_SUCCESS, MPI_ERR_COUNT
 * (too many sources or too many bytes), MPI_ERR_TYPE, MPI_ERR_OP, MPI_ERR_ARG
 * (null pointer) or MPI_ERR_OTHER (CUDA error). */
int cail_reduce_sources_noalloc(const void *const *srcs, int nsrc, void *dst, size_t count,
                                MPI_Datatype datatype, MPI_Op op, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CAIL_NOALLOC_H */
