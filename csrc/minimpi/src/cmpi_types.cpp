// cmpi_types.cpp — datatype table and host reduction operators of minimpi.
//
// Integer SUM and PROD are evaluated in the unsigned type of the same width,
// so overflow wraps (two's complement) instead of being undefined; this is
// the bit pattern every GPU kernel in this repository produces as well.
// MAX/MIN keep the C expression (a > b) ? a : b with the accumulator on the
// left, which fixes the NaN behaviour for floating point.
#include "cmpi_internal.h"

#include <type_traits>
#include <vector>

namespace cmpi {

namespace {

std::vector<TypeInfo> &table() {
    static std::vector<TypeInfo> t = [] {
        std::vector<TypeInfo> v(0x100);
        auto def = [&](MPI_Datatype h, int size, Kind k) {
            TypeInfo &ti = v[h];
            ti.valid = ti.predefined = ti.committed = true;
            ti.size = size;
            ti.kind = k;
            ti.base = h;
            ti.base_count = 1;
        };
        Kind klong = sizeof(long) == 8 ? K_I64 : K_I32;
        Kind kulong = sizeof(long) == 8 ? K_U64 : K_U32;
        def(MPI_CHAR, 1, K_I8);
        def(MPI_SIGNED_CHAR, 1, K_I8);
        def(MPI_UNSIGNED_CHAR, 1, K_U8);
        def(MPI_BYTE, 1, K_U8);
        def(MPI_SHORT, 2, K_I16);
        def(MPI_UNSIGNED_SHORT, 2, K_U16);
        def(MPI_INT, 4, K_I32);
        def(MPI_UNSIGNED, 4, K_U32);
        def(MPI_LONG, (int)sizeof(long), klong);
        def(MPI_UNSIGNED_LONG, (int)sizeof(unsigned long), kulong);
        def(MPI_LONG_LONG, 8, K_I64);
        def(MPI_LONG_LONG_INT, 8, K_I64);
        def(MPI_UNSIGNED_LONG_LONG, 8, K_U64);
        def(MPI_FLOAT, 4, K_F32);
        def(MPI_DOUBLE, 8, K_F64);
        def(MPI_LONG_DOUBLE, (int)sizeof(long double), K_LD);
        def(MPI_INT8_T, 1, K_I8);
        def(MPI_UINT8_T, 1, K_U8);
        def(MPI_INT16_T, 2, K_I16);
        def(MPI_UINT16_T, 2, K_U16);
        def(MPI_INT32_T, 4, K_I32);
        def(MPI_UINT32_T, 4, K_U32);
        def(MPI_INT64_T, 8, K_I64);
        def(MPI_UINT64_T, 8, K_U64);
        def(MPI_C_BOOL, 1, K_BOOL);
        def(MPI_WCHAR, (int)sizeof(wchar_t), K_WCHAR);
        def(MPI_AINT, (int)sizeof(MPI_Aint), K_I64);
        def(MPI_COUNT, (int)sizeof(MPI_Count), K_I64);
        def(MPI_2INT, 8, K_2INT);
        return v;
    }();
    return t;
}

template <typename T> struct Unsigned { using type = typename std::make_unsigned<T>::type; };

template <typename T, bool IsInt = std::is_integral<T>::value>
struct Arith {
    static T add(T a, T b) { return a + b; }
    static T mul(T a, T b) { return a * b; }
};
// Wrapping arithmetic in an unsigned type no narrower than unsigned int (8-
// and 16-bit unsigned operands would be promoted to signed int).
template <typename T>
struct Arith<T, true> {
    using U = typename Unsigned<T>::type;
    using W = typename std::conditional<(sizeof(U) < sizeof(unsigned)), unsigned, U>::type;
    static T add(T a, T b) { return (T)(U)((W)(U)a + (W)(U)b); }
    static T mul(T a, T b) { return (T)(U)((W)(U)a * (W)(U)b); }
};

template <typename T>
int reduce_t(const T *in, T *io, long long n, MPI_Op op) {
    switch (op) {
    case MPI_SUM: for (long long i = 0; i < n; ++i) io[i] = Arith<T>::add(io[i], in[i]); return MPI_SUCCESS;
    case MPI_PROD: for (long long i = 0; i < n; ++i) io[i] = Arith<T>::mul(io[i], in[i]); return MPI_SUCCESS;
    case MPI_MAX: for (long long i = 0; i < n; ++i) io[i] = (io[i] > in[i]) ? io[i] : in[i]; return MPI_SUCCESS;
    case MPI_MIN: for (long long i = 0; i < n; ++i) io[i] = (io[i] < in[i]) ? io[i] : in[i]; return MPI_SUCCESS;
    case MPI_REPLACE: for (long long i = 0; i < n; ++i) io[i] = in[i]; return MPI_SUCCESS;
    case MPI_NO_OP: return MPI_SUCCESS;
    default: break;
    }
    if constexpr (std::is_integral<T>::value) {
        switch (op) {
        case MPI_LAND: for (long long i = 0; i < n; ++i) io[i] = (T)(io[i] && in[i]); return MPI_SUCCESS;
        case MPI_LOR: for (long long i = 0; i < n; ++i) io[i] = (T)(io[i] || in[i]); return MPI_SUCCESS;
        case MPI_LXOR: for (long long i = 0; i < n; ++i) io[i] = (T)(!io[i] != !in[i]); return MPI_SUCCESS;
        case MPI_BAND: for (long long i = 0; i < n; ++i) io[i] = (T)(io[i] & in[i]); return MPI_SUCCESS;
        case MPI_BOR: for (long long i = 0; i < n; ++i) io[i] = (T)(io[i] | in[i]); return MPI_SUCCESS;
        case MPI_BXOR: for (long long i = 0; i < n; ++i) io[i] = (T)(io[i] ^ in[i]); return MPI_SUCCESS;
        default: break;
        }
    }
    return MPI_ERR_OP;
}

int reduce_bool(const bool *in, bool *io, long long n, MPI_Op op) {
    switch (op) {
    case MPI_LAND: for (long long i = 0; i < n; ++i) io[i] = io[i] && in[i]; return MPI_SUCCESS;
    case MPI_LOR: for (long long i = 0; i < n; ++i) io[i] = io[i] || in[i]; return MPI_SUCCESS;
    case MPI_LXOR: for (long long i = 0; i < n; ++i) io[i] = io[i] != in[i]; return MPI_SUCCESS;
    case MPI_REPLACE: for (long long i = 0; i < n; ++i) io[i] = in[i]; return MPI_SUCCESS;
    case MPI_NO_OP: return MPI_SUCCESS;
    default: return MPI_ERR_OP;
    }
}

}  // namespace

const TypeInfo *type_info(MPI_Datatype dt) {
    auto &t = table();
    if (dt <= 0 || (size_t)dt >= t.size() || !t[dt].valid) return nullptr;
    return &t[dt];
}

int type_new_contiguous(int count, MPI_Datatype old, MPI_Datatype *out) {
    const TypeInfo *o = type_info(old);
    if (!o || count < 0) return MPI_ERR_TYPE;
    TypeInfo ti;
    ti.valid = true;
    ti.size = o->size * count;
    ti.kind = o->kind;
    ti.base_count = o->base_count * count;
    ti.base = o->base;
    auto &t = table();
    for (size_t i = 0x100; i < t.size(); ++i) {
        if (!t[i].valid) { t[i] = ti; *out = (MPI_Datatype)i; return MPI_SUCCESS; }
    }
    t.push_back(ti);
    *out = (MPI_Datatype)(t.size() - 1);
    return MPI_SUCCESS;
}

int type_free(MPI_Datatype *dt) {
    auto &t = table();
    if (!dt || *dt < 0x100 || (size_t)*dt >= t.size() || !t[*dt].valid) return MPI_ERR_TYPE;
    t[*dt] = TypeInfo{};
    *dt = MPI_DATATYPE_NULL;
    return MPI_SUCCESS;
}

bool op_valid(MPI_Op op) { return op >= MPI_MAX && op <= MPI_NO_OP; }

int reduce_host(const void *in, void *io, long long n, Kind kind, MPI_Op op) {
    switch (kind) {
    case K_I8: return reduce_t((const int8_t *)in, (int8_t *)io, n, op);
    case K_U8: return reduce_t((const uint8_t *)in, (uint8_t *)io, n, op);
    case K_I16: return reduce_t((const int16_t *)in, (int16_t *)io, n, op);
    case K_U16: return reduce_t((const uint16_t *)in, (uint16_t *)io, n, op);
    case K_I32: return reduce_t((const int32_t *)in, (int32_t *)io, n, op);
    case K_U32: return reduce_t((const uint32_t *)in, (uint32_t *)io, n, op);
    case K_I64: return reduce_t((const int64_t *)in, (int64_t *)io, n, op);
    case K_U64: return reduce_t((const uint64_t *)in, (uint64_t *)io, n, op);
    case K_F32: return reduce_t((const float *)in, (float *)io, n, op);
    case K_F64: return reduce_t((const double *)in, (double *)io, n, op);
    case K_LD: return reduce_t((const long double *)in, (long double *)io, n, op);
    case K_BOOL: return reduce_bool((const bool *)in, (bool *)io, n, op);
    case K_WCHAR: return reduce_t((const wchar_t *)in, (wchar_t *)io, n, op);
    default: return MPI_ERR_OP;
    }
}

}  // namespace cmpi
