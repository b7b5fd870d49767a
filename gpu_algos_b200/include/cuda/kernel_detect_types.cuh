// cuda/kernel_detect_types.cuh -- element types of a kernel's tensors and the
// relative tolerance the driver checks them with.
//
// A kernel class may name NumberA/B/C/D/Temp/Internal; absent names default
// to Kernel::Number.  The tolerance is 2^-(precision_bits - tol_bits) with
// precision 11 bits for half, 24 for float, 53 for double, exact (0) for
// integers; for several types the least precise one (largest epsilon) sets
// it, and an exact integer type defers to any floating-point one
// (include/cuda/kernel_detect_types.cuh:74-173 in gpu_algos).
#pragma once

#include <cmath>
#include <concepts>
#include <string>
#include <type_traits>

#include "cuda/type_traits.cuh"

namespace detect {

#define GLMB_DETECT_NUMBER(X)                                              \
    template <typename K>                                                  \
    concept has_Number##X = requires { typename K::Number##X; };           \
    template <typename K>                                                  \
    struct Number##X##_of {                                                \
        using type = typename K::Number;                                   \
    };                                                                     \
    template <has_Number##X K>                                             \
    struct Number##X##_of<K> {                                             \
        using type = typename K::Number##X;                                \
    };                                                                     \
    template <typename K>                                                  \
    using Number##X = typename Number##X##_of<K>::type;

GLMB_DETECT_NUMBER(A)
GLMB_DETECT_NUMBER(B)
GLMB_DETECT_NUMBER(C)
GLMB_DETECT_NUMBER(D)
GLMB_DETECT_NUMBER(Temp)
GLMB_DETECT_NUMBER(Internal)
#undef GLMB_DETECT_NUMBER

// Type the errors are computed in: the output type (D for 3-in kernels),
// double for integer kernels.
template <typename K>
struct NumberE_of {
    using type = std::conditional_t<std::is_integral_v<typename K::Number>, double, typename K::Number>;
};
template <has_NumberD K>
struct NumberE_of<K> {
    using type = typename K::NumberD;
};
template <typename K>
using NumberE = typename NumberE_of<K>::type;

template <typename T>
struct Precision {
    static constexpr int bits = std::is_same_v<T, __half> ? 11
                                : std::is_same_v<T, float> ? 24
                                : std::is_same_v<T, double> ? 53
                                                            : 0;
    static constexpr bool exact = std::is_integral_v<T>;
};

template <typename... Ts>
struct Tolerance;

template <typename T>
struct Tolerance<T> {
    using type = T;
    static constexpr int precision_bits = Precision<T>::exact ? int(8 * sizeof(T)) : Precision<T>::bits;
    static constexpr float precision = Precision<T>::exact ? 0.0f : float(1.0 / double(1ull << Precision<T>::bits));
    static std::string name() {
        if constexpr (std::is_same_v<T, __half>) return "CUDA __half";
        else if constexpr (std::is_same_v<T, float>) return "float";
        else if constexpr (std::is_same_v<T, double>) return "double";
        else if constexpr (std::is_unsigned_v<T>) return "unsigned integer";
        else return "signed integer";
    }
    static float tolerance(const int lost_precision_bits) {
        if constexpr (Precision<T>::exact) return 0.0f;
        else return float(std::pow(0.5, Precision<T>::bits - lost_precision_bits));
    }
};

// Several types: the one with the largest epsilon decides.
template <typename T1, typename T2, typename... Ts>
struct Tolerance<T1, T2, Ts...>
    : Tolerance<std::conditional_t<(Tolerance<T1>::precision >= Tolerance<T2>::precision), T1, T2>, Ts...> {};

template <typename K>
struct Numbers {
    using A = NumberA<K>;
    using B = NumberB<K>;
    using C = NumberC<K>;
    using D = NumberD<K>;
    using Temp = NumberTemp<K>;
    using Internal = NumberInternal<K>;
    using E = NumberE<K>;
    using Tolerance = detect::Tolerance<A, B, C, D, Temp, Internal>;
};

}  // namespace detect
