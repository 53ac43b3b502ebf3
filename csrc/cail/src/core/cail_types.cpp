// cail_types.cpp — MPI handle <-> element type / operator mapping.
//
// Accepts the 23 handles the reference accepts (src/core/cail_types.c:5-31
// there): the 20 documented datatypes plus the aliases MPI_SIGNED_CHAR,
// MPI_BYTE and MPI_LONG_LONG_INT.  MPI handles are not integral constants in
// every MPI, so the mapping is a chain of comparisons, as it must be.
#include "cail_types.h"

extern "C" {

cail_datatype_t cail_mpi_type_to_dtype(MPI_Datatype dt) {
    if (dt == MPI_CHAR || dt == MPI_SIGNED_CHAR || dt == MPI_INT8_T) return CAIL_CHAR;
    if (dt == MPI_UNSIGNED_CHAR || dt == MPI_BYTE || dt == MPI_UINT8_T) return CAIL_UCHAR;
    if (dt == MPI_SHORT || dt == MPI_INT16_T) return CAIL_SHORT;
    if (dt == MPI_UNSIGNED_SHORT || dt == MPI_UINT16_T) return CAIL_USHORT;
    if (dt == MPI_INT || dt == MPI_INT32_T) return CAIL_INT;
    if (dt == MPI_UNSIGNED || dt == MPI_UINT32_T) return CAIL_UINT;
    if (dt == MPI_LONG) return CAIL_LONG;
    if (dt == MPI_UNSIGNED_LONG) return CAIL_ULONG;
    if (dt == MPI_LONG_LONG || dt == MPI_LONG_LONG_INT || dt == MPI_INT64_T) return CAIL_LONG_LONG;
    if (dt == MPI_UNSIGNED_LONG_LONG || dt == MPI_UINT64_T) return CAIL_ULONGLONG;
    if (dt == MPI_FLOAT) return CAIL_FLOAT;
    if (dt == MPI_DOUBLE) return CAIL_DOUBLE;
    return CAIL_INVALID;
}

cail_op_t cail_mpi_op_to_optype(MPI_Op op) {
    if (op == MPI_SUM) return CAIL_SUM;
    if (op == MPI_PROD) return CAIL_PROD;
    if (op == MPI_MAX) return CAIL_MAX;
    if (op == MPI_MIN) return CAIL_MIN;
    return CAIL_OP_INVALID;
}

MPI_Datatype cail_dtype_to_mpi_type(cail_datatype_t d) {
    switch (d) {
    case CAIL_CHAR: return MPI_CHAR;
    case CAIL_INT: return MPI_INT;
    case CAIL_LONG: return MPI_LONG;
    case CAIL_FLOAT: return MPI_FLOAT;
    case CAIL_DOUBLE: return MPI_DOUBLE;
    case CAIL_LONG_LONG: return MPI_LONG_LONG;
    case CAIL_UCHAR: return MPI_UNSIGNED_CHAR;
    case CAIL_UINT: return MPI_UNSIGNED;
    case CAIL_ULONG: return MPI_UNSIGNED_LONG;
    case CAIL_ULONGLONG: return MPI_UNSIGNED_LONG_LONG;
    case CAIL_SHORT: return MPI_SHORT;
    case CAIL_USHORT: return MPI_UNSIGNED_SHORT;
    default: return MPI_DATATYPE_NULL;
    }
}

MPI_Op cail_optype_to_mpi_op(cail_op_t op) {
    switch (op) {
    case CAIL_SUM: return MPI_SUM;
    case CAIL_PROD: return MPI_PROD;
    case CAIL_MAX: return MPI_MAX;
    case CAIL_MIN: return MPI_MIN;
    default: return MPI_OP_NULL;
    }
}

int cail_type_supported(MPI_Datatype dt) { return cail_mpi_type_to_dtype(dt) != CAIL_INVALID; }
int cail_op_supported(MPI_Op op) { return cail_mpi_op_to_optype(op) != CAIL_OP_INVALID; }

int cail_type_size(cail_datatype_t d) {
    switch (d) {
    case CAIL_CHAR: case CAIL_UCHAR: return 1;
    case CAIL_SHORT: case CAIL_USHORT: return 2;
    case CAIL_INT: case CAIL_UINT: case CAIL_FLOAT: return 4;
    case CAIL_LONG: case CAIL_ULONG: return (int)sizeof(long);
    case CAIL_LONG_LONG: case CAIL_ULONGLONG: case CAIL_DOUBLE: return 8;
    default: return 0;
    }
}

cail_elem_class_t cail_elem_class(cail_datatype_t d) {
    switch (d) {
    case CAIL_CHAR: return CAIL_EC_I8;
    case CAIL_UCHAR: return CAIL_EC_U8;
    case CAIL_SHORT: return CAIL_EC_I16;
    case CAIL_USHORT: return CAIL_EC_U16;
    case CAIL_INT: return CAIL_EC_I32;
    case CAIL_UINT: return CAIL_EC_U32;
    case CAIL_LONG: return sizeof(long) == 8 ? CAIL_EC_I64 : CAIL_EC_I32;
    case CAIL_ULONG: return sizeof(long) == 8 ? CAIL_EC_U64 : CAIL_EC_U32;
    case CAIL_LONG_LONG: return CAIL_EC_I64;
    case CAIL_ULONGLONG: return CAIL_EC_U64;
    case CAIL_FLOAT: return CAIL_EC_F32;
    case CAIL_DOUBLE: return CAIL_EC_F64;
    default: return CAIL_EC_NUM;
    }
}

const char *cail_dtype_name(cail_datatype_t d) {
    static const char *names[] = {"CHAR", "INT", "LONG", "FLOAT", "DOUBLE", "LONG_LONG",
                                  "UCHAR", "UINT", "ULONG", "ULONGLONG", "SHORT", "USHORT"};
    return (d >= 0 && d < CAIL_NUM_DTYPES) ? names[d] : "UNKNOWN";
}

const char *cail_op_name(cail_op_t op) {
    static const char *names[] = {"SUM", "PROD", "MAX", "MIN"};
    return (op >= 0 && op < CAIL_NUM_OPS) ? names[op] : "UNKNOWN";
}

const char *cail_algo_name(int a) {
    static const char *names[] = {"recursive_doubling", "ring", "rabenseifner",
                                  "one_shot", "two_shot", "nvls", "ce_two_shot", "copy"};
    if (a == CAIL_ALGO_AUTO) return "auto";
    return (a >= 0 && a < CAIL_NUM_ALGOS) ? names[a] : "unknown";
}

const char *cail_mpi_type_name(MPI_Datatype dt) {
    struct { MPI_Datatype h; const char *n; } tbl[] = {
        {MPI_CHAR, "MPI_CHAR"}, {MPI_SIGNED_CHAR, "MPI_CHAR"},
        {MPI_UNSIGNED_CHAR, "MPI_UNSIGNED_CHAR"}, {MPI_BYTE, "MPI_UNSIGNED_CHAR"},
        {MPI_SHORT, "MPI_SHORT"}, {MPI_UNSIGNED_SHORT, "MPI_UNSIGNED_SHORT"},
        {MPI_INT, "MPI_INT"}, {MPI_UNSIGNED, "MPI_UNSIGNED"}, {MPI_LONG, "MPI_LONG"},
        {MPI_UNSIGNED_LONG, "MPI_UNSIGNED_LONG"}, {MPI_LONG_LONG, "MPI_LONG_LONG"},
        {MPI_LONG_LONG_INT, "MPI_LONG_LONG"}, {MPI_UNSIGNED_LONG_LONG, "MPI_UNSIGNED_LONG_LONG"},
        {MPI_FLOAT, "MPI_FLOAT"}, {MPI_DOUBLE, "MPI_DOUBLE"}, {MPI_INT8_T, "MPI_INT8_T"},
        {MPI_UINT8_T, "MPI_UINT8_T"}, {MPI_INT16_T, "MPI_INT16_T"},
        {MPI_UINT16_T, "MPI_UINT16_T"}, {MPI_INT32_T, "MPI_INT32_T"},
        {MPI_UINT32_T, "MPI_UINT32_T"}, {MPI_INT64_T, "MPI_INT64_T"},
        {MPI_UINT64_T, "MPI_UINT64_T"},
    };
    for (auto &e : tbl)
        if (e.h == dt) return e.n;
    return "UNKNOWN";
}

const char *cail_mpi_op_name(MPI_Op op) {
    if (op == MPI_SUM) return "MPI_SUM";
    if (op == MPI_PROD) return "MPI_PROD";
    if (op == MPI_MAX) return "MPI_MAX";
    if (op == MPI_MIN) return "MPI_MIN";
    return "UNKNOWN";
}

}  // extern "C"
