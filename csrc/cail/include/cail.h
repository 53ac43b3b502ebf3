/*
 * cail.h — cail-b200 public header.
 *
 * cail-b200 is a transparent MPI_Allreduce interposition library: load it
 * with LD_PRELOAD, or link it before -lmpi, and every MPI_Allreduce on
 * device buffers that it supports runs on its Blackwell NVLink kernels;
 * everything else reaches the MPI library through PMPI_Allreduce.  No API
 * call is needed.
 *
 * The functions below are optional extensions for tools and benchmarks
 * (they are what the reference's header leaves empty, cail.h:14-18 there).
 */
#ifndef CAIL_H
#define CAIL_H

#include <mpi.h>
#include <stddef.h>

#define CAIL_VERSION_MAJOR 0
#define CAIL_VERSION_MINOR 1
#define CAIL_VERSION_PATCH 0

#ifdef __cplusplus
extern "C" {
#endif

/* Library version string, e.g. "0.1.0 (cuda sm_100a)" or "0.1.0 (host)". */
const char *cail_version(void);

/* Name of the algorithm that ran the last intercepted MPI_Allreduce of this
 * process ("one_shot", "two_shot", "nvls", "ce_two_shot", "copy" (a one-rank
 * communicator on device buffers),
 * "recursive_doubling", "ring", "rabenseifner", "pmpi" for a passthrough,
 * "none" before the first call). */
const char *cail_last_algorithm(void);

/* Counters since initialisation. */
typedef struct cail_stats {
    unsigned long long calls;          /* MPI_Allreduce calls seen */
    unsigned long long passthrough;    /* calls forwarded to PMPI_Allreduce */
    unsigned long long by_algo[12];    /* calls per algorithm, index 1 + (0 recursive_doubling, 1 ring,
                                          2 rabenseifner, 3 one_shot, 4 two_shot, 5 nvls,
                                          6 ce_two_shot, 7 copy); index 0 and 9..11 unused */
    unsigned long long bytes;          /* payload bytes reduced by cail algorithms */
    unsigned long long reg_hits;       /* registration cache hits (peer buffers) */
    unsigned long long reg_misses;     /* registration cache misses (IPC opens) */
    unsigned long long device_errors;  /* device collectives that reported an error */
    unsigned long long launches;       /* CUDA kernels launched by cail */
} cail_stats_t;
int cail_get_stats(cail_stats_t *out);

/* 1 if communicator `comm` runs cail's NVLink kernels (after its first
 * device MPI_Allreduce), 0 if it uses the point-to-point algorithms. */
int cail_comm_uses_nvlink(MPI_Comm comm);

/* 1 if NVLS (NVSwitch multicast) is active on `comm`, else 0. */
int cail_comm_uses_nvls(MPI_Comm comm);

/* Stream ordering of device calls.  1 (default, env CAIL_STREAM_SYNC): cail
 * first waits for all work already queued on the legacy default stream,
 * which covers a cudaMemcpy from pageable memory whose DMA may still be in
 * flight when it returns.  0: the caller guarantees that the buffers are
 * complete (e.g. it synchronised the producing stream), which lets cail's
 * kernels overlap later work on other streams.  Returns the previous mode. */
int cail_set_stream_sync(int mode);

/* Completion of device calls on NVLink communicators.
 * 0 (default, env CAIL_STREAM_ORDERED): MPI_Allreduce returns when the result
 * is in the receive buffer, as MPI specifies.  1: one_shot, two_shot and nvls
 * calls return once their kernel is queued and the legacy default stream has
 * been made to wait for it, the completion semantics of NCCL: work queued
 * later on the legacy stream (and cudaMemcpy, cudaDeviceSynchronize) sees the
 * result, host reads of the buffer without such a synchronisation do not.
 * Two-shot calls then run the push kernel, which needs no host barrier (the
 * zero-copy kernel, used otherwise, synchronises the host).  Needs stream sync
 * mode 1; ce_two_shot stays host-synchronous.  A device-side timeout of a
 * stream-ordered call is reported by the next call or at MPI_Finalize.
 * Returns the previous mode. */
int cail_set_stream_ordered(int mode);

/* The algorithm auto mode picks for an intercepted device-buffer call of
 * `bytes` bytes on an NVLink communicator of `nranks` ranks, under this
 * process' environment (CAIL_ONESHOT_MAX, CAIL_MSG_SMALL_THRESHOLD,
 * CAIL_TUNE_FILE, CAIL_NVLS_MIN_RANKS, CAIL_NVLS_MIN, CAIL_CE_MIN,
 * CAIL_NVLS), assuming an NVSwitch fabric with multicast.  NULL for an unsupported type or op.  Needs
 * no MPI_Init: for checking a tuning before a job. */
const char *cail_nvlink_auto_algorithm(int nranks, size_t bytes, MPI_Datatype datatype, MPI_Op op);

#ifdef __cplusplus
}
#endif

#endif /* CAIL_H */
