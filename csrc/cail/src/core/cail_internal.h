// cail_internal.h — process-wide state, configuration and logging of cail.
//
// Logging keeps the reference's three levels and prefixes
// (src/core/cail_internal.h:17-27 there): "[cail] ..." when CAIL_DEBUG is
// on, "[cail WARN] ..." unless CAIL_WARN=0, "[cail ERROR] ..." always.  Every
// warning goes through CAIL_WARN, including the GPU backend's (the
// reference's CUDA backend printed its warnings unconditionally).
#pragma once

#include <mpi.h>
#include <stddef.h>
#include <stdio.h>

#include "cail.h"
#include "cail_types.h"

#define CAIL_DBG(fmt, ...) \
    do { if (cail_global_state.debug) fprintf(stderr, "[cail] " fmt "\n", ##__VA_ARGS__); } while (0)
#define CAIL_ERR(fmt, ...) fprintf(stderr, "[cail ERROR] " fmt "\n", ##__VA_ARGS__)
#define CAIL_WARN(fmt, ...) \
    do { if (cail_global_state.warn) fprintf(stderr, "[cail WARN] " fmt "\n", ##__VA_ARGS__); } while (0)
#define CAIL_CHECK(rc) do { if ((rc) != MPI_SUCCESS) return (rc); } while (0)

// Environment variables of the reference contract.
#define CAIL_ENV_DEBUG "CAIL_DEBUG"
#define CAIL_ENV_ALGO "CAIL_ALGO"
#define CAIL_ENV_MSG_SMALL_THRESHOLD "CAIL_MSG_SMALL_THRESHOLD"
#define CAIL_ENV_NPROCS_THRESHOLD "CAIL_NPROCS_THRESHOLD"
#define CAIL_ENV_MIN_MSG_SIZE "CAIL_MIN_MSG_SIZE"
#define CAIL_ENV_WARN "CAIL_WARN"
// cail-b200 additions.
#define CAIL_ENV_DEVICE_TIMEOUT_MS "CAIL_DEVICE_TIMEOUT_MS"
#define CAIL_ENV_NVLS "CAIL_NVLS"
#define CAIL_ENV_ONESHOT_MAX "CAIL_ONESHOT_MAX"
#define CAIL_ENV_TUNE_FILE "CAIL_TUNE_FILE"
#define CAIL_ENV_STATS "CAIL_STATS"
#define CAIL_ENV_TRACE "CAIL_TRACE"
#define CAIL_ENV_FLUSH_RECV "CAIL_FLUSH_RECV"
#define CAIL_ENV_STREAM_SYNC "CAIL_STREAM_SYNC"
#define CAIL_ENV_STREAM_ORDERED "CAIL_STREAM_ORDERED"
#define CAIL_ENV_DEVICE_CHECKS "CAIL_DEVICE_CHECKS"

#define CAIL_DEFAULT_MSG_SMALL_THRESHOLD 262144U /* 256 KiB */
#define CAIL_DEFAULT_NPROCS_THRESHOLD 4U
#define CAIL_DEFAULT_MIN_MSG_SIZE 32768U /* 32 KiB */
#define CAIL_DEFAULT_DEVICE_TIMEOUT_MS 10000L

/* Largest power of two <= n (n > 0). */
static inline int cail_pof2(int n) {
    int p = 1;
    while (p <= n / 2) p <<= 1;
    return p;
}
static inline int cail_is_pof2(int n) { return n > 0 && (n & (n - 1)) == 0; }

typedef struct cail_state {
    int initialized;
    int debug;
    int warn;
    size_t msg_small_threshold;
    int msg_small_threshold_set; /* the user set CAIL_MSG_SMALL_THRESHOLD */
    int nprocs_threshold;        /* parsed for compatibility; no dispatch rule uses it */
    size_t min_msg_size;
    int force_algo;
    long device_timeout_ms;
    int nvls;                    /* 0 off, 1 use when the fabric supports it */
    size_t oneshot_max;          /* NVLink one-shot/two-shot crossover in bytes, 0 = tuned */
    int flush_recv;
    int stats;
    FILE *trace;
    int stream_sync;             /* order device work after the legacy stream */
    int profile;                 /* CAIL_PROFILE: host-side phase timers */
    int stream_ordered;          /* one-shot calls complete in stream order, not on the host */
    int nvtx;                    /* CAIL_NVTX: an NVTX range per call (CUDA build) */
    int device_checks;           /* CAIL_DEVICE_CHECKS: kernels validate their arguments and bounds */
} cail_state_t;

/* Opt-in host-side phase timers (CAIL_PROFILE=1), averaged per call and
 * printed at MPI_Finalize. */
enum {
    CAIL_PH_FILTER = 0,  /* shim: entry to dispatch (type/op/pointer checks) */
    CAIL_PH_SETUP,       /* dispatch + context lookup + argument preparation */
    CAIL_PH_LAUNCH,      /* kernel launch calls */
    CAIL_PH_WAIT,        /* waiting for the kernels (stream synchronise) */
    CAIL_PH_HOSTSYNC,    /* host barriers of the two-shot path */
    CAIL_PH_TOTAL,       /* whole intercepted call */
    CAIL_PH_N
};

#ifdef __cplusplus
extern "C" {
#endif

/* One line of CAIL_TUNE_FILE: measured crossovers for NVLink communicators of
 * `nranks` ranks, in bytes; -1 where the line gives none.  The environment
 * variables of the same meaning (CAIL_ONESHOT_MAX, CAIL_MSG_SMALL_THRESHOLD,
 * CAIL_NVLS_MIN_RANKS / CAIL_NVLS_MIN, CAIL_CE_MIN) take precedence. */
typedef struct {
    int nranks;
    long long oneshot_max; /* one_shot up to this size */
    long long nvls_min;    /* nvls from this size (where multimem can reduce the pair) */
    long long ce_min;      /* ce_two_shot from this size */
} cail_tune_t;

/* The CAIL_TUNE_FILE line for `nranks`, or NULL. */
const cail_tune_t *cail_tune_for(int nranks);

extern cail_state_t cail_global_state;
extern cail_stats_t cail_counters;
extern int cail_last_algo;
extern double cail_prof_us[CAIL_PH_N];
extern unsigned long long cail_prof_calls;

/* Adds now - t0 to phase ph of the current call when profiling; returns now
 * (or t0 when off).  cail_prof_end_call() closes the call. */
double cail_prof_mark(int ph, double t0);
void cail_prof_end_call(double total_us);

int cail_init(MPI_Comm comm);
void cail_load_config(void);
void cail_finalize(void);
int cail_is_initialized(void);

int cail_allreduce_dispatch(const void *sendbuf, void *recvbuf, int count, MPI_Datatype datatype,
                            MPI_Op op, MPI_Comm comm);

int cail_buf_get_tmp(void **ptr, size_t size);
void cail_buf_release_tmp(void *ptr);
void cail_buf_finalize(void);

/* Per-call trace line (CAIL_TRACE=path): algo,bytes,count,dtype,op,nprocs,usec */
void cail_trace_call(int algo, size_t bytes, int count, cail_datatype_t dt, cail_op_t op,
                     int nprocs, double usec);
double cail_now_us(void);

#ifdef __cplusplus
}
#endif
