// cail_pmpi.cpp — the interposed MPI_Allreduce and MPI_Finalize.
//
// Filter order and messages are the reference's contract
// (src/core/cail_pmpi.c:19-86 there):
//   lazy init (abort on failure) -> count == 0 -> unsupported type (WARN)
//   -> unsupported op (WARN) -> intercommunicator (DBG) -> host buffers
//   (DBG; not in the host-only build) -> msg < CAIL_MIN_MSG_SIZE (DBG)
//   -> dispatch; a dispatch error falls back to PMPI_Allreduce (DBG).
// One deliberate difference: an error reported by an NVLink kernel is
// returned to the caller ([cail ERROR]) instead of being retried through
// PMPI_Allreduce, because the failed collective may have partially updated
// peers' buffers and the ranks may disagree about what happened.
#include "../core/cail_internal.h"
#include "../dev/cail_dev.h"
#include "../gpu/cail_gpu.h"

#ifndef CAIL_HOST_PATH
#include <nvtx3/nvToolsExt.h>  // header-only; calls are no-ops without a profiler attached
#endif

extern "C" int cail_allreduce_dispatch_ex(const void *sendbuf, void *recvbuf, int count,
                                          MPI_Datatype datatype, MPI_Op op, MPI_Comm comm,
                                          int *may_fallback);

namespace {
inline int passthrough(const void *s, void *r, int n, MPI_Datatype dt, MPI_Op op, MPI_Comm comm) {
    cail_last_algo = -3;
    cail_counters.passthrough++;
    return PMPI_Allreduce(s, r, n, dt, op, comm);
}
}  // namespace

namespace {

int allreduce_filtered(const void *sendbuf, void *recvbuf, int count, MPI_Datatype datatype, MPI_Op op,
                       MPI_Comm comm) {
    int rc;
    if (!cail_is_initialized()) {
        rc = cail_init(comm);
        if (rc != MPI_SUCCESS) {
            CAIL_ERR("cail_init failed (rc=%d), aborting", rc);
            PMPI_Abort(comm, rc);
        }
    }
    cail_counters.calls++;
    const double t_in = cail_global_state.profile ? cail_now_us() : 0.0;
    if (count == 0) return MPI_SUCCESS;

    if (!cail_type_supported(datatype)) {
        CAIL_WARN("falling back to PMPI_Allreduce: unsupported type=%s", cail_mpi_type_name(datatype));
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }
    if (!cail_op_supported(op)) {
        CAIL_WARN("falling back to PMPI_Allreduce: unsupported op=%s", cail_mpi_op_name(op));
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }
    int is_inter = 0;
    PMPI_Comm_test_inter(comm, &is_inter);
    if (is_inter) {
        CAIL_DBG("falling back to PMPI_Allreduce: intercommunicator");
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }
#ifndef CAIL_HOST_PATH
    if (!cail_gpu_is_device_pointer(recvbuf)) {
        CAIL_DBG("falling back to PMPI_Allreduce: recvbuf is not on GPU");
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }
    if (sendbuf != MPI_IN_PLACE && !cail_gpu_is_device_pointer(sendbuf)) {
        CAIL_DBG("falling back to PMPI_Allreduce: sendbuf is not on GPU");
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }
#endif
    int type_size = 0;
    PMPI_Type_size(datatype, &type_size);
    size_t msg_size = (size_t)count * (size_t)type_size;
    if (msg_size < cail_global_state.min_msg_size) {
        CAIL_DBG("falling back to PMPI_Allreduce: msg_size=%zu < min_msg_size=%zu", msg_size,
                 cail_global_state.min_msg_size);
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }

    double t0 = cail_global_state.trace ? cail_now_us() : 0.0;
    cail_prof_mark(CAIL_PH_FILTER, t_in);
    int may_fallback = 1;
    rc = cail_allreduce_dispatch_ex(sendbuf, recvbuf, count, datatype, op, comm, &may_fallback);
    if (cail_global_state.profile) cail_prof_end_call(cail_now_us() - t_in);
    if (rc != MPI_SUCCESS) {
        if (!may_fallback) {
            CAIL_ERR("device allreduce failed (rc=%d); not retrying through PMPI", rc);
            return rc;
        }
        CAIL_DBG("cail_allreduce_dispatch failed (rc=%d), falling back to PMPI", rc);
        return passthrough(sendbuf, recvbuf, count, datatype, op, comm);
    }
    if (cail_global_state.trace) {
        int np = 1;
        PMPI_Comm_size(comm, &np);
        cail_trace_call(cail_last_algo, msg_size, count, cail_mpi_type_to_dtype(datatype),
                        cail_mpi_op_to_optype(op), np, cail_now_us() - t0);
    }
    return MPI_SUCCESS;
}

}  // namespace

extern "C" {

int MPI_Allreduce(const void *sendbuf, void *recvbuf, int count, MPI_Datatype datatype, MPI_Op op,
                  MPI_Comm comm) {
#ifndef CAIL_HOST_PATH
    // CAIL_NVTX=1: one range per call, named with the message size, and a
    // mark with the algorithm that ran (or "pmpi")
    cail_load_config();
    const bool nvtx = cail_global_state.nvtx != 0;
    if (nvtx) {
        int ts = 0;
        PMPI_Type_size(datatype, &ts);
        char msg[96];
        snprintf(msg, sizeof msg, "cail MPI_Allreduce %lld B", (long long)count * ts);
        nvtxRangePushA(msg);
    }
#endif
    const int rc = allreduce_filtered(sendbuf, recvbuf, count, datatype, op, comm);
    // the call ran on its buffers' device; the caller keeps its own
    cail_gpu_restore_device();
#ifndef CAIL_HOST_PATH
    if (nvtx) {
        char msg[64];
        snprintf(msg, sizeof msg, "cail algorithm=%s", cail_last_algorithm());
        nvtxMarkA(msg);
        nvtxRangePop();
    }
#endif
    return rc;
}

int MPI_Finalize(void) {
#ifndef CAIL_HOST_PATH
    cail_dev_finalize_all();
#endif
    cail_finalize();
    return PMPI_Finalize();
}

int cail_comm_uses_nvlink(MPI_Comm comm);
int cail_comm_uses_nvls(MPI_Comm comm);

}  // extern "C"
