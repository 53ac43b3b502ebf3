/*
 * mpi.h — minimpi: the single-node MPI subset bundled with cail-b200.
 *
 * Neither the development machine nor the GPU hosts ship an MPI library, and
 * cail is by contract a PMPI interposer that sits on top of one.  minimpi is
 * the MPI underneath: every routine exists twice, as a strong PMPI_x symbol
 * and as a weak MPI_x alias of it, exactly like production MPIs, so that a
 * library loaded first (LD_PRELOAD or link order) can define MPI_x and reach
 * the real implementation through PMPI_x.
 *
 * Scope: one node, one process per rank, shared-memory transport.  Device
 * (CUDA) buffers are accepted everywhere ("CUDA-aware"): point-to-point moves
 * them with a CUDA-IPC rendezvous (the receiver copies straight out of the
 * sender's allocation), collectives stage them through host memory.
 *
 * Handles are plain ints, as in MPICH-derived MPIs.  The set of routines is
 * what the reference test programs, the cail interposer (topology probe,
 * attribute caching) and this repository's tests need.
 */
#ifndef MINIMPI_MPI_H
#define MINIMPI_MPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MINIMPI 1
#define MPI_VERSION 3
#define MPI_SUBVERSION 1

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Op;
typedef int MPI_Request;
typedef int MPI_Errhandler;
typedef int MPI_Group;
typedef long MPI_Aint;
typedef long long MPI_Count;
typedef long long MPI_Offset;

typedef struct MPI_Status {
    int MPI_SOURCE;
    int MPI_TAG;
    int MPI_ERROR;
    int cancelled;
    long long nbytes; /* received payload in bytes (MPI_Get_count divides) */
} MPI_Status;

/* ---- error classes ---------------------------------------------------- */
#define MPI_SUCCESS          0
#define MPI_ERR_BUFFER       1
#define MPI_ERR_COUNT        2
#define MPI_ERR_TYPE         3
#define MPI_ERR_TAG          4
#define MPI_ERR_COMM         5
#define MPI_ERR_RANK         6
#define MPI_ERR_REQUEST      7
#define MPI_ERR_ROOT         8
#define MPI_ERR_GROUP        9
#define MPI_ERR_OP          10
#define MPI_ERR_TOPOLOGY    11
#define MPI_ERR_DIMS        12
#define MPI_ERR_ARG         13
#define MPI_ERR_UNKNOWN     14
#define MPI_ERR_TRUNCATE    15
#define MPI_ERR_OTHER       16
#define MPI_ERR_INTERN      17
#define MPI_ERR_IN_STATUS   18
#define MPI_ERR_PENDING     19
#define MPI_ERR_KEYVAL      48
#define MPI_ERR_NO_MEM      34
#define MPI_ERR_PROC_FAILED 75  /* a peer process exited or timed out */
#define MPI_ERR_LASTCODE    127

/* ---- special values ---------------------------------------------------- */
#define MPI_IN_PLACE        ((void *)-1)
#define MPI_BOTTOM          ((void *)0)
#define MPI_STATUS_IGNORE   ((MPI_Status *)0)
#define MPI_STATUSES_IGNORE ((MPI_Status *)0)
#define MPI_ANY_SOURCE      (-2)
#define MPI_ANY_TAG         (-1)
#define MPI_PROC_NULL       (-1)
#define MPI_UNDEFINED       (-32766)
#define MPI_TAG_UB_VALUE    (1 << 28)
#define MPI_MAX_PROCESSOR_NAME 256
#define MPI_MAX_ERROR_STRING   256
#define MPI_MAX_LIBRARY_VERSION_STRING 256

#define MPI_THREAD_SINGLE     0
#define MPI_THREAD_FUNNELED   1
#define MPI_THREAD_SERIALIZED 2
#define MPI_THREAD_MULTIPLE   3

/* ---- communicators ---------------------------------------------------- */
#define MPI_COMM_NULL   ((MPI_Comm)0)
#define MPI_COMM_WORLD  ((MPI_Comm)1)
#define MPI_COMM_SELF   ((MPI_Comm)2)
#define MPI_REQUEST_NULL ((MPI_Request)0)
#define MPI_ERRHANDLER_NULL ((MPI_Errhandler)0)
#define MPI_ERRORS_ARE_FATAL ((MPI_Errhandler)1)
#define MPI_ERRORS_RETURN    ((MPI_Errhandler)2)

/* ---- datatypes ---------------------------------------------------------
 * Every named type has its own handle, aliases included (MPI_INT32_T is not
 * MPI_INT), because interposers map them one by one.  Values below 0x100
 * are predefined; derived (contiguous) types are allocated above it. */
#define MPI_DATATYPE_NULL       ((MPI_Datatype)0)
#define MPI_CHAR                ((MPI_Datatype)1)
#define MPI_SIGNED_CHAR         ((MPI_Datatype)2)
#define MPI_UNSIGNED_CHAR       ((MPI_Datatype)3)
#define MPI_BYTE                ((MPI_Datatype)4)
#define MPI_SHORT               ((MPI_Datatype)5)
#define MPI_UNSIGNED_SHORT      ((MPI_Datatype)6)
#define MPI_INT                 ((MPI_Datatype)7)
#define MPI_UNSIGNED            ((MPI_Datatype)8)
#define MPI_LONG                ((MPI_Datatype)9)
#define MPI_UNSIGNED_LONG       ((MPI_Datatype)10)
#define MPI_LONG_LONG           ((MPI_Datatype)11)
#define MPI_LONG_LONG_INT       ((MPI_Datatype)12)
#define MPI_UNSIGNED_LONG_LONG  ((MPI_Datatype)13)
#define MPI_FLOAT               ((MPI_Datatype)14)
#define MPI_DOUBLE              ((MPI_Datatype)15)
#define MPI_LONG_DOUBLE         ((MPI_Datatype)16)
#define MPI_INT8_T              ((MPI_Datatype)17)
#define MPI_UINT8_T             ((MPI_Datatype)18)
#define MPI_INT16_T             ((MPI_Datatype)19)
#define MPI_UINT16_T            ((MPI_Datatype)20)
#define MPI_INT32_T             ((MPI_Datatype)21)
#define MPI_UINT32_T            ((MPI_Datatype)22)
#define MPI_INT64_T             ((MPI_Datatype)23)
#define MPI_UINT64_T            ((MPI_Datatype)24)
#define MPI_C_BOOL              ((MPI_Datatype)25)
#define MPI_WCHAR               ((MPI_Datatype)26)
#define MPI_AINT                ((MPI_Datatype)27)
#define MPI_COUNT               ((MPI_Datatype)28)
#define MPI_2INT                ((MPI_Datatype)29)

/* ---- reduction operations ----------------------------------------------- */
#define MPI_OP_NULL  ((MPI_Op)0)
#define MPI_MAX      ((MPI_Op)1)
#define MPI_MIN      ((MPI_Op)2)
#define MPI_SUM      ((MPI_Op)3)
#define MPI_PROD     ((MPI_Op)4)
#define MPI_LAND     ((MPI_Op)5)
#define MPI_BAND     ((MPI_Op)6)
#define MPI_LOR      ((MPI_Op)7)
#define MPI_BOR      ((MPI_Op)8)
#define MPI_LXOR     ((MPI_Op)9)
#define MPI_BXOR     ((MPI_Op)10)
#define MPI_REPLACE  ((MPI_Op)11)
#define MPI_NO_OP    ((MPI_Op)12)

/* ---- attribute caching -------------------------------------------------- */
typedef int MPI_Comm_copy_attr_function(MPI_Comm, int, void *, void *, void *, int *);
typedef int MPI_Comm_delete_attr_function(MPI_Comm, int, void *, void *);
#define MPI_COMM_NULL_COPY_FN   ((MPI_Comm_copy_attr_function *)0)
#define MPI_COMM_NULL_DELETE_FN ((MPI_Comm_delete_attr_function *)0)
#define MPI_KEYVAL_INVALID (-1)
#define MPI_TAG_UB 0x64400001

/* ---- prototypes: each routine as MPI_x (weak) and PMPI_x (strong) ------- */
#define MINIMPI_DECL(ret, name, args) ret MPI_##name args; ret PMPI_##name args;

MINIMPI_DECL(int, Init, (int *argc, char ***argv))
MINIMPI_DECL(int, Init_thread, (int *argc, char ***argv, int required, int *provided))
MINIMPI_DECL(int, Initialized, (int *flag))
MINIMPI_DECL(int, Finalized, (int *flag))
MINIMPI_DECL(int, Finalize, (void))
MINIMPI_DECL(int, Query_thread, (int *provided))
MINIMPI_DECL(int, Abort, (MPI_Comm comm, int errorcode))
MINIMPI_DECL(double, Wtime, (void))
MINIMPI_DECL(double, Wtick, (void))
MINIMPI_DECL(int, Get_processor_name, (char *name, int *resultlen))
MINIMPI_DECL(int, Get_library_version, (char *version, int *resultlen))
MINIMPI_DECL(int, Error_string, (int errorcode, char *string, int *resultlen))

MINIMPI_DECL(int, Comm_rank, (MPI_Comm comm, int *rank))
MINIMPI_DECL(int, Comm_size, (MPI_Comm comm, int *size))
MINIMPI_DECL(int, Comm_test_inter, (MPI_Comm comm, int *flag))
MINIMPI_DECL(int, Comm_dup, (MPI_Comm comm, MPI_Comm *newcomm))
MINIMPI_DECL(int, Comm_split, (MPI_Comm comm, int color, int key, MPI_Comm *newcomm))
MINIMPI_DECL(int, Comm_free, (MPI_Comm *comm))
MINIMPI_DECL(int, Comm_set_errhandler, (MPI_Comm comm, MPI_Errhandler errhandler))
MINIMPI_DECL(int, Comm_create_keyval, (MPI_Comm_copy_attr_function *copy_fn,
                                       MPI_Comm_delete_attr_function *delete_fn,
                                       int *keyval, void *extra_state))
MINIMPI_DECL(int, Comm_free_keyval, (int *keyval))
MINIMPI_DECL(int, Comm_set_attr, (MPI_Comm comm, int keyval, void *attribute_val))
MINIMPI_DECL(int, Comm_get_attr, (MPI_Comm comm, int keyval, void *attribute_val, int *flag))
MINIMPI_DECL(int, Comm_delete_attr, (MPI_Comm comm, int keyval))

MINIMPI_DECL(int, Type_size, (MPI_Datatype datatype, int *size))
MINIMPI_DECL(int, Type_get_extent, (MPI_Datatype datatype, MPI_Aint *lb, MPI_Aint *extent))
MINIMPI_DECL(int, Type_contiguous, (int count, MPI_Datatype oldtype, MPI_Datatype *newtype))
MINIMPI_DECL(int, Type_commit, (MPI_Datatype *datatype))
MINIMPI_DECL(int, Type_free, (MPI_Datatype *datatype))
MINIMPI_DECL(int, Get_count, (const MPI_Status *status, MPI_Datatype datatype, int *count))

MINIMPI_DECL(int, Send, (const void *buf, int count, MPI_Datatype datatype, int dest, int tag,
                         MPI_Comm comm))
MINIMPI_DECL(int, Recv, (void *buf, int count, MPI_Datatype datatype, int source, int tag,
                         MPI_Comm comm, MPI_Status *status))
MINIMPI_DECL(int, Sendrecv, (const void *sendbuf, int sendcount, MPI_Datatype sendtype,
                             int dest, int sendtag, void *recvbuf, int recvcount,
                             MPI_Datatype recvtype, int source, int recvtag, MPI_Comm comm,
                             MPI_Status *status))
MINIMPI_DECL(int, Isend, (const void *buf, int count, MPI_Datatype datatype, int dest, int tag,
                          MPI_Comm comm, MPI_Request *request))
MINIMPI_DECL(int, Irecv, (void *buf, int count, MPI_Datatype datatype, int source, int tag,
                          MPI_Comm comm, MPI_Request *request))
MINIMPI_DECL(int, Wait, (MPI_Request *request, MPI_Status *status))
MINIMPI_DECL(int, Waitall, (int count, MPI_Request requests[], MPI_Status statuses[]))
MINIMPI_DECL(int, Test, (MPI_Request *request, int *flag, MPI_Status *status))

MINIMPI_DECL(int, Barrier, (MPI_Comm comm))
MINIMPI_DECL(int, Bcast, (void *buffer, int count, MPI_Datatype datatype, int root, MPI_Comm comm))
MINIMPI_DECL(int, Reduce, (const void *sendbuf, void *recvbuf, int count, MPI_Datatype datatype,
                           MPI_Op op, int root, MPI_Comm comm))
MINIMPI_DECL(int, Allreduce, (const void *sendbuf, void *recvbuf, int count,
                              MPI_Datatype datatype, MPI_Op op, MPI_Comm comm))
MINIMPI_DECL(int, Reduce_local, (const void *inbuf, void *inoutbuf, int count,
                                 MPI_Datatype datatype, MPI_Op op))
MINIMPI_DECL(int, Allgather, (const void *sendbuf, int sendcount, MPI_Datatype sendtype,
                              void *recvbuf, int recvcount, MPI_Datatype recvtype,
                              MPI_Comm comm))
MINIMPI_DECL(int, Gather, (const void *sendbuf, int sendcount, MPI_Datatype sendtype,
                           void *recvbuf, int recvcount, MPI_Datatype recvtype, int root,
                           MPI_Comm comm))

#undef MINIMPI_DECL

/* ---- minimpi extensions (MPIX_) ----------------------------------------
 * MPIX_Comm_set_test_inter marks a communicator as an intercommunicator for
 * MPI_Comm_test_inter only.  minimpi has no real intercommunicators; the
 * flag lets a test drive an interposer's intercommunicator branch. */
int MPIX_Comm_set_test_inter(MPI_Comm comm, int flag);
/* Host identity used by topology probes: a stable hash of the node name. */
unsigned long long MPIX_Node_id(void);

#ifdef __cplusplus
}
#endif

#endif /* MINIMPI_MPI_H */
