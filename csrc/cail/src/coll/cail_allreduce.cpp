// cail_allreduce.cpp — algorithm selection.
//
// Forced mode (CAIL_ALGO) keeps the reference's behaviour for its three
// algorithms (src/coll/allreduce/cail_allreduce.c:99-136 there): a
// compiled-out algorithm is an [cail ERROR] and PMPI_Abort; Rabenseifner with
// count < pof2 warns and falls back to PMPI_Allreduce.  The NVLink
// algorithms can be forced too; when the communicator cannot run them the
// call warns and falls back, and a forced nvls on a (type, op) pair that
// multimem cannot reduce runs two_shot instead.
//
// Auto mode:
//   * NVLink communicator (cail_dev_comm_get != nullptr): one_shot up to the
//     tuned crossover (or CAIL_MSG_SMALL_THRESHOLD when the user set it),
//     then nvls when the fabric and the (type, op) pair allow it, else
//     two_shot;
//   * otherwise the reference's rule (cail_allreduce.c:140-157 there):
//     count < pof2 -> small; threshold halved for non-power-of-two P >= 16;
//     msg < threshold -> recursive doubling, else Rabenseifner.
#include "../core/cail_internal.h"
#include "../dev/cail_dev.h"
#include "../gpu/cail_gpu.h"
#include "cail_p2p_algos.h"

namespace {

typedef int (*algo_fn)(const void *, void *, int, MPI_Datatype, MPI_Op, MPI_Comm);

struct P2PAlgo {
    int id;
    const char *name;
    algo_fn fn;  // nullptr when compiled out
};

const P2PAlgo &p2p_algo(int id) {
    static const P2PAlgo tbl[] = {
#ifdef CAIL_ENABLE_RECURSIVE_DOUBLING
        {CAIL_ALGO_RECURSIVE_DOUBLING, "recursive_doubling", cail_allreduce_recursive_doubling},
#else
        {CAIL_ALGO_RECURSIVE_DOUBLING, "recursive_doubling", nullptr},
#endif
#ifdef CAIL_ENABLE_RING
        {CAIL_ALGO_RING, "ring", cail_allreduce_ring},
#else
        {CAIL_ALGO_RING, "ring", nullptr},
#endif
#ifdef CAIL_ENABLE_RABENSEIFNER
        {CAIL_ALGO_RABENSEIFNER, "rabenseifner", cail_allreduce_rabenseifner},
#else
        {CAIL_ALGO_RABENSEIFNER, "rabenseifner", nullptr},
#endif
    };
    return tbl[id];
}

void count_algo(int algo, size_t bytes) {
    cail_last_algo = algo;
    cail_counters.by_algo[algo + 1]++;
    cail_counters.bytes += bytes;
}

// Auto-mode call of a point-to-point algorithm: WARN + PMPI when compiled out.
int call_auto(int id, const char *reason, const void *s, void *r, int n, MPI_Datatype dt, MPI_Op op,
              MPI_Comm comm, size_t bytes) {
    const P2PAlgo &a = p2p_algo(id);
    if (!a.fn) {
        CAIL_WARN("%s selected (%s) but disabled at compile time, falling back to PMPI", a.name,
                  reason);
        cail_last_algo = -3;
        cail_counters.passthrough++;
        return PMPI_Allreduce(s, r, n, dt, op, comm);
    }
    CAIL_DBG("algorithm=%s (%s)", a.name, reason);
    count_algo(id, bytes);
    return a.fn(s, r, n, dt, op, comm);
}

}  // namespace

extern "C" int cail_allreduce_dispatch_ex(const void *sendbuf, void *recvbuf, int count,
                                          MPI_Datatype datatype, MPI_Op op, MPI_Comm comm,
                                          int *may_fallback) {
    *may_fallback = 1;
    cail_datatype_t dtype = cail_mpi_type_to_dtype(datatype);
    cail_op_t optype = cail_mpi_op_to_optype(op);
    (void)optype;  // used by the NVLink path only
    size_t msg = (size_t)count * (size_t)cail_type_size(dtype);
    int nprocs;
    PMPI_Comm_size(comm, &nprocs);
    int pof2 = cail_pof2(nprocs);
    int forced = cail_global_state.force_algo;

    // ---- forced: the reference's algorithms
    if (forced == CAIL_ALGO_RECURSIVE_DOUBLING || forced == CAIL_ALGO_RING ||
        forced == CAIL_ALGO_RABENSEIFNER) {
        const P2PAlgo &a = p2p_algo(forced);
        if (!a.fn) {
            CAIL_ERR("CAIL_ALGO=%s forced but disabled at compile time, aborting", a.name);
            PMPI_Abort(comm, MPI_ERR_INTERN);
            return MPI_ERR_INTERN;
        }
        if (forced == CAIL_ALGO_RABENSEIFNER && count < pof2) {
            CAIL_WARN("forced rabenseifner but count=%d < pof2=%d, falling back to PMPI", count, pof2);
            cail_last_algo = -3;
            cail_counters.passthrough++;
            return PMPI_Allreduce(sendbuf, recvbuf, count, datatype, op, comm);
        }
        CAIL_DBG("algorithm=%s (forced)", a.name);
        count_algo(forced, msg);
        return a.fn(sendbuf, recvbuf, count, datatype, op, comm);
    }

    // ---- one rank: the result is the input.  The reference's three
    // algorithms copy sendbuf to recvbuf and return when P == 1
    // (cail_allreduce_recursive_doubling.c:52-58 there); here the copy runs
    // without any communicator setup, and an in-place call does nothing.
#ifndef CAIL_HOST_PATH
    if (nprocs == 1) {
        CAIL_DBG("algorithm=%s (one rank)", cail_algo_name(CAIL_ALGO_COPY));
        count_algo(CAIL_ALGO_COPY, msg);
        const void *src = sendbuf == MPI_IN_PLACE ? recvbuf : sendbuf;
        return cail_gpu_single_rank(src, recvbuf, msg) == 0 ? MPI_SUCCESS : MPI_ERR_OTHER;
    }
#endif

    // ---- NVLink device path
#ifndef CAIL_HOST_PATH
    struct cail_dev_comm *dc = cail_dev_comm_get(comm);
    if (cail_algo_is_device(forced)) {
        if (!dc) {
            CAIL_WARN("forced %s but the communicator has no NVLink path, falling back to PMPI",
                      cail_algo_name(forced));
            cail_last_algo = -3;
            cail_counters.passthrough++;
            return PMPI_Allreduce(sendbuf, recvbuf, count, datatype, op, comm);
        }
        int algo = forced;
        if (algo == CAIL_ALGO_NVLS && !cail_dev_nvls_ok(dc, dtype, optype)) {
            CAIL_DBG("nvls cannot reduce %s %s here, using two_shot", cail_dtype_name(dtype),
                     cail_op_name(optype));
            algo = CAIL_ALGO_TWO_SHOT;
        }
        CAIL_DBG("algorithm=%s (forced)", cail_algo_name(algo));
        count_algo(algo, msg);
        *may_fallback = 0;
        int rc = cail_dev_allreduce(dc, algo, sendbuf, recvbuf, count, dtype, optype);
        if (rc != MPI_SUCCESS) cail_counters.device_errors++;
        return rc;
    }
    if (dc) {
        int algo = cail_dev_pick_algo(dc, msg, count, dtype, optype);
        CAIL_DBG("algorithm=%s (nvlink auto, msg_size=%zu)", cail_algo_name(algo), msg);
        count_algo(algo, msg);
        *may_fallback = 0;
        int rc = cail_dev_allreduce(dc, algo, sendbuf, recvbuf, count, dtype, optype);
        if (rc != MPI_SUCCESS) cail_counters.device_errors++;
        return rc;
    }
#else
    if (cail_algo_is_device(forced)) {
        CAIL_WARN("forced %s needs the CUDA build, falling back to PMPI", cail_algo_name(forced));
        cail_last_algo = -3;
        cail_counters.passthrough++;
        return PMPI_Allreduce(sendbuf, recvbuf, count, datatype, op, comm);
    }
#endif

    // ---- auto: the reference's decision table
    if (count < pof2)
        return call_auto(CAIL_ALGO_RECURSIVE_DOUBLING, "count < pof2", sendbuf, recvbuf, count,
                         datatype, op, comm, msg);
    size_t effective_small = cail_global_state.msg_small_threshold;
    if (!cail_is_pof2(nprocs) && nprocs >= 16) effective_small /= 2;
    if (msg < effective_small)
        return call_auto(CAIL_ALGO_RECURSIVE_DOUBLING, "msg_size < msg_small_threshold", sendbuf,
                         recvbuf, count, datatype, op, comm, msg);
    return call_auto(CAIL_ALGO_RABENSEIFNER, "msg_size >= msg_small_threshold", sendbuf, recvbuf,
                     count, datatype, op, comm, msg);
}

extern "C" int cail_allreduce_dispatch(const void *sendbuf, void *recvbuf, int count,
                                       MPI_Datatype datatype, MPI_Op op, MPI_Comm comm) {
    int may_fallback;
    return cail_allreduce_dispatch_ex(sendbuf, recvbuf, count, datatype, op, comm, &may_fallback);
}
