// cail_types.h — element types, reduction operators and algorithm ids.
//
// The 12 element types and 4 operators are the contract of the reference
// (src/core/cail_types.h:12-43 there); 23 MPI datatype handles map onto the
// 12 types (cail_types.cpp).  Unlike the reference, the device kernels are
// not indexed by this enum: they are instantiated per storage class (width,
// signedness, float), see cail_elem_class().
#pragma once

#include <mpi.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    CAIL_CHAR = 0,
    CAIL_INT = 1,
    CAIL_LONG = 2,
    CAIL_FLOAT = 3,
    CAIL_DOUBLE = 4,
    CAIL_LONG_LONG = 5,
    CAIL_UCHAR = 6,
    CAIL_UINT = 7,
    CAIL_ULONG = 8,
    CAIL_ULONGLONG = 9,
    CAIL_SHORT = 10,
    CAIL_USHORT = 11,
    CAIL_NUM_DTYPES,
    CAIL_INVALID = -1
} cail_datatype_t;

typedef enum {
    CAIL_SUM = 0,
    CAIL_PROD = 1,
    CAIL_MAX = 2,
    CAIL_MIN = 3,
    CAIL_NUM_OPS,
    CAIL_OP_INVALID = -1
} cail_op_t;

/* Algorithms.  The first three are the reference's (host-driven, over PMPI
 * point-to-point); the others are cail-b200's NVLink paths. */
typedef enum {
    CAIL_ALGO_AUTO = -1,
    CAIL_ALGO_RECURSIVE_DOUBLING = 0,
    CAIL_ALGO_RING = 1,
    CAIL_ALGO_RABENSEIFNER = 2,
    CAIL_ALGO_ONE_SHOT = 3,
    CAIL_ALGO_TWO_SHOT = 4,
    CAIL_ALGO_NVLS = 5,
    CAIL_ALGO_CE_TWO_SHOT = 6,
    CAIL_ALGO_COPY = 7,          /* one-rank communicator: dst = src, chosen automatically */
    CAIL_NUM_ALGOS = 8
} cail_algo_t;

/* Storage classes the kernels are instantiated for. */
typedef enum {
    CAIL_EC_I8 = 0, CAIL_EC_U8, CAIL_EC_I16, CAIL_EC_U16, CAIL_EC_I32, CAIL_EC_U32,
    CAIL_EC_I64, CAIL_EC_U64, CAIL_EC_F32, CAIL_EC_F64, CAIL_EC_NUM
} cail_elem_class_t;

/* 1 for the algorithms that run on the NVLink device path. */
static inline int cail_algo_is_device(int a) {
    return a == CAIL_ALGO_ONE_SHOT || a == CAIL_ALGO_TWO_SHOT || a == CAIL_ALGO_NVLS ||
           a == CAIL_ALGO_CE_TWO_SHOT;
}

cail_datatype_t cail_mpi_type_to_dtype(MPI_Datatype dt);
cail_op_t cail_mpi_op_to_optype(MPI_Op op);
MPI_Datatype cail_dtype_to_mpi_type(cail_datatype_t dtype);
MPI_Op cail_optype_to_mpi_op(cail_op_t op);

int cail_type_supported(MPI_Datatype dt);
int cail_op_supported(MPI_Op op);
int cail_type_size(cail_datatype_t dt);
cail_elem_class_t cail_elem_class(cail_datatype_t dt);

const char *cail_mpi_type_name(MPI_Datatype dt);
const char *cail_mpi_op_name(MPI_Op op);
const char *cail_dtype_name(cail_datatype_t dt);
const char *cail_op_name(cail_op_t op);
const char *cail_algo_name(int algo);

#ifdef __cplusplus
}
#endif
