// cail_dev.h — the NVLink (single-node, peer-accessible GPUs) collectives.
//
// A communicator whose ranks all sit on one node, each on its own GPU with
// peer access to every other, gets a device context on its first device
// MPI_Allreduce (collective setup: topology probe, IPC workspace exchange,
// optional NVLS multicast object).  The algorithms below then run as single
// sm_100a kernels that read and write peer GPUs' memory directly:
//   one_shot     every rank pushes its data to all ranks' scratch and folds
//                the P copies in rank order;
//   two_shot     rank r reduces slice r from all ranks and writes it to all;
//   nvls         two-shot through NVSwitch multicast (multimem.ld_reduce/st);
//   ce_two_shot  two-shot with the transfers on the copy engines.
#pragma once

#include <mpi.h>
#include <stddef.h>

#include "../core/cail_types.h"

struct cail_dev_comm;

#ifdef __cplusplus
extern "C" {
#endif

/* Device context of `comm`, created collectively on first use.  Returns
 * nullptr (on every rank alike) when the NVLink path cannot serve `comm`. */
struct cail_dev_comm *cail_dev_comm_get(MPI_Comm comm);

/* Algorithm for an auto-dispatched call of `bytes` bytes on a device comm. */
int cail_dev_pick_algo(struct cail_dev_comm *dc, size_t bytes, int count, cail_datatype_t dt,
                       cail_op_t op);

/* 1 if NVLS can reduce (dt, op) on this communicator. */
int cail_dev_nvls_ok(struct cail_dev_comm *dc, cail_datatype_t dt, cail_op_t op);

/* Runs algo (ONE_SHOT, TWO_SHOT, NVLS or CE_TWO_SHOT).  Returns MPI_SUCCESS, or an error
 * after which no fallback is possible (the collective may be partial). */
int cail_dev_allreduce(struct cail_dev_comm *dc, int algo, const void *sendbuf, void *recvbuf,
                       int count, cail_datatype_t dt, cail_op_t op);

/* Tears down every device context (MPI_Finalize). */
void cail_dev_finalize_all(void);

#ifdef __cplusplus
}
#endif
