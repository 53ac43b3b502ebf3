// cail_p2p_algos.h — the host-driven PMPI point-to-point algorithms.
#pragma once

#include <mpi.h>

#ifdef __cplusplus
extern "C" {
#endif

int cail_allreduce_recursive_doubling(const void *sendbuf, void *recvbuf, int count,
                                      MPI_Datatype datatype, MPI_Op op, MPI_Comm comm);
int cail_allreduce_ring(const void *sendbuf, void *recvbuf, int count, MPI_Datatype datatype,
                        MPI_Op op, MPI_Comm comm);
int cail_allreduce_rabenseifner(const void *sendbuf, void *recvbuf, int count,
                                MPI_Datatype datatype, MPI_Op op, MPI_Comm comm);

#ifdef __cplusplus
}
#endif
