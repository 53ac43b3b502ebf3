// cail_ops.h — the four reduction operators, defined once for host and device.
//
//   SUM, PROD : integers wrap (computed in the unsigned type of the same
//               width, so signed overflow is defined); floats are IEEE.
//   MAX, MIN  : (acc > x) ? acc : x  and  (acc < x) ? acc : x, accumulator on
//               the left — the reference's expressions
//               (src/gpu/cuda/cail_cuda_reduce.cu:24-42 there), which fix
//               which operand wins when a NaN is involved.
// Every kernel and every host loop of cail-b200 folds values in rank order
// acc = x_0; acc = op(acc, x_1); ...  with these functions, and minimpi's
// PMPI_Allreduce does the same, so integer results are bit-identical and
// the P2P float results are too.
#pragma once

#include <stdint.h>

#include <type_traits>

#include "../core/cail_types.h"

#if defined(__CUDACC__)
#define CAIL_HD __host__ __device__ __forceinline__
#else
#define CAIL_HD inline
#endif

namespace cail {

template <typename T, bool I = std::is_integral<T>::value>
struct Wrap {
    static CAIL_HD T add(T a, T b) { return a + b; }
    static CAIL_HD T mul(T a, T b) { return a * b; }
};
// Integers wrap: the arithmetic runs in an unsigned type at least as wide as
// unsigned int, since 8- and 16-bit unsigned operands would otherwise be
// promoted to (signed) int, where 65535 * 65535 overflows.
template <typename T>
struct Wrap<T, true> {
    using U = typename std::make_unsigned<T>::type;
    using W = typename std::conditional<(sizeof(U) < sizeof(unsigned)), unsigned, U>::type;
    static CAIL_HD T add(T a, T b) { return (T)(U)((W)(U)a + (W)(U)b); }
    static CAIL_HD T mul(T a, T b) { return (T)(U)((W)(U)a * (W)(U)b); }
};

template <int OP, typename T>
CAIL_HD T apply(T acc, T x) {
    if constexpr (OP == CAIL_SUM) return Wrap<T>::add(acc, x);
    else if constexpr (OP == CAIL_PROD) return Wrap<T>::mul(acc, x);
    else if constexpr (OP == CAIL_MAX) return (acc > x) ? acc : x;
    else return (acc < x) ? acc : x;
}

// Element storage class -> C type.
template <int EC> struct EcType;
template <> struct EcType<CAIL_EC_I8> { using T = int8_t; };
template <> struct EcType<CAIL_EC_U8> { using T = uint8_t; };
template <> struct EcType<CAIL_EC_I16> { using T = int16_t; };
template <> struct EcType<CAIL_EC_U16> { using T = uint16_t; };
template <> struct EcType<CAIL_EC_I32> { using T = int32_t; };
template <> struct EcType<CAIL_EC_U32> { using T = uint32_t; };
template <> struct EcType<CAIL_EC_I64> { using T = int64_t; };
template <> struct EcType<CAIL_EC_U64> { using T = uint64_t; };
template <> struct EcType<CAIL_EC_F32> { using T = float; };
template <> struct EcType<CAIL_EC_F64> { using T = double; };

// SUM and PROD do not depend on signedness (wrapping arithmetic), so the
// kernels for them are instantiated for the unsigned class only.
constexpr int canonical_class(int op, int ec) {
    if (op == CAIL_SUM || op == CAIL_PROD) {
        switch (ec) {
        case CAIL_EC_I8: return CAIL_EC_U8;
        case CAIL_EC_I16: return CAIL_EC_U16;
        case CAIL_EC_I32: return CAIL_EC_U32;
        case CAIL_EC_I64: return CAIL_EC_U64;
        default: return ec;
        }
    }
    return ec;
}

// Calls f.template operator()<OP, EC>() for the runtime (op, ec) pair.
// Returns false when the pair is out of range.
template <typename F>
bool dispatch_op_class(int op, int ec, F &&f) {
    auto by_class = [&](auto opc) -> bool {
        constexpr int OP = decltype(opc)::value;
        switch (canonical_class(OP, ec)) {
        case CAIL_EC_I8: f.template operator()<OP, CAIL_EC_I8>(); return true;
        case CAIL_EC_U8: f.template operator()<OP, CAIL_EC_U8>(); return true;
        case CAIL_EC_I16: f.template operator()<OP, CAIL_EC_I16>(); return true;
        case CAIL_EC_U16: f.template operator()<OP, CAIL_EC_U16>(); return true;
        case CAIL_EC_I32: f.template operator()<OP, CAIL_EC_I32>(); return true;
        case CAIL_EC_U32: f.template operator()<OP, CAIL_EC_U32>(); return true;
        case CAIL_EC_I64: f.template operator()<OP, CAIL_EC_I64>(); return true;
        case CAIL_EC_U64: f.template operator()<OP, CAIL_EC_U64>(); return true;
        case CAIL_EC_F32: f.template operator()<OP, CAIL_EC_F32>(); return true;
        case CAIL_EC_F64: f.template operator()<OP, CAIL_EC_F64>(); return true;
        default: return false;
        }
    };
    switch (op) {
    case CAIL_SUM: return by_class(std::integral_constant<int, CAIL_SUM>{});
    case CAIL_PROD: return by_class(std::integral_constant<int, CAIL_PROD>{});
    case CAIL_MAX: return by_class(std::integral_constant<int, CAIL_MAX>{});
    case CAIL_MIN: return by_class(std::integral_constant<int, CAIL_MIN>{});
    default: return false;
    }
}

}  // namespace cail
