// cuda/type_traits.cuh -- element types the GLM kernel classes accept.
//
// CUDA_scalar: the 8/16/32/64-bit integers, float, double and __half -- the
// type set of the reference (include/cuda/type_traits.cuh:25-72 in gpu_algos).
#pragma once

#include <cstdint>
#include <type_traits>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

template <typename T>
constexpr bool is_CUDA_integer_v =
    std::is_integral_v<T> && !std::is_same_v<T, bool> &&
    (sizeof(T) == 1 || sizeof(T) == 2 || sizeof(T) == 4 || sizeof(T) == 8);

template <typename T>
constexpr bool is_CUDA_floating_point_v = std::is_floating_point_v<T> || std::is_same_v<T, __half>;

template <typename T>
concept CUDA_integer = is_CUDA_integer_v<T>;

template <typename T>
concept CUDA_floating_point = is_CUDA_floating_point_v<T>;

template <typename T>
concept CUDA_scalar = is_CUDA_integer_v<T> || is_CUDA_floating_point_v<T>;

template <CUDA_scalar T>
using Printable_Number = std::conditional_t<std::is_same_v<T, __half>, float, T>;

template <CUDA_scalar Number>
constexpr bool is_positive(const Number value) {
    if constexpr (std::is_same_v<Number, __half>) return __half2float(value) > 0.0f;
    else return value > Number(0);
}

template <CUDA_scalar Number>
constexpr bool is_negative(const Number value) {
    if constexpr (std::is_same_v<Number, __half>) return __half2float(value) < 0.0f;
    else if constexpr (std::is_unsigned_v<Number>) return false;
    else return value < Number(0);
}
