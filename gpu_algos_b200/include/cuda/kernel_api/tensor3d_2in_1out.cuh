// cuda/kernel_api/tensor3d_2in_1out.cuh -- compile-time contract of a kernel
// with two Tensor3D inputs (A, B), one output C and a temp (the reference's
// TENSOR3D_KERNEL_2IN_1OUT, include/cuda/kernel_api/tensor3d_2in_1out.cuh:32-137
// in gpu_algos).
#pragma once

#include <concepts>
#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#include "common/types/tensor3d.hpp"
#include "cuda/kernel_detect_types.cuh"
#include "cuda/type_traits.cuh"

template <typename S>
concept TENSOR3D_KERNEL_SPEC_2IN_1OUT = requires(S spec) {
    { spec.n_rows_A_ } -> std::same_as<const long&>;
    { spec.n_cols_A_ } -> std::same_as<const long&>;
    { spec.n_sheets_A_ } -> std::same_as<const long&>;
    { spec.n_rows_B_ } -> std::same_as<const long&>;
    { spec.n_cols_B_ } -> std::same_as<const long&>;
    { spec.n_sheets_B_ } -> std::same_as<const long&>;
    { spec.n_rows_C_ } -> std::same_as<const long&>;
    { spec.n_cols_C_ } -> std::same_as<const long&>;
    { spec.n_sheets_C_ } -> std::same_as<const long&>;
    { spec.n_rows_temp_ } -> std::same_as<const long&>;
    { spec.n_cols_temp_ } -> std::same_as<const long&>;
    { spec.n_sheets_temp_ } -> std::same_as<const long&>;
    { dim3(spec.block_dim_) } -> std::same_as<dim3>;
    { dim3(spec.grid_dim_) } -> std::same_as<dim3>;
};

template <typename S>
struct Check_tensor3d_kernel_spec_2In_1Out {
    static_assert(TENSOR3D_KERNEL_SPEC_2IN_1OUT<S>, "not a valid TENSOR3D_KERNEL_SPEC_2IN_1OUT");
    static constexpr bool check_passed = true;
};

template <typename K>
concept TENSOR3D_KERNEL_2IN_1OUT = requires(K kernel) {
    typename K::Number;
    typename K::Kernel_spec;
    requires TENSOR3D_KERNEL_SPEC_2IN_1OUT<typename K::Kernel_spec>;
    { kernel.spec_ } -> std::same_as<const typename K::Kernel_spec&>;
    { kernel.run_device_kernel(std::declval<const typename detect::Numbers<K>::A*>(),
                               std::declval<const typename detect::Numbers<K>::B*>(),
                               std::declval<typename detect::Numbers<K>::C*>(),
                               std::declval<typename detect::Numbers<K>::Temp*>(),
                               std::declval<cudaStream_t>()) } -> std::same_as<void>;
    { kernel.run_host_kernel(std::declval<const Tensor3D<typename detect::Numbers<K>::A>&>(),
                             std::declval<const Tensor3D<typename detect::Numbers<K>::B>&>()) }
        -> std::same_as<Tensor3D<typename detect::Numbers<K>::C>>;
};

template <typename K>
struct Check_tensor3d_kernel_2In_1Out {
    static_assert(TENSOR3D_KERNEL_2IN_1OUT<K>, "not a valid TENSOR3D_KERNEL_2IN_1OUT");
    static constexpr bool check_passed = true;
};

template <template <CUDA_scalar> class Kernel>
struct Check_tensor3d_kernel_2In_1Out_template {
    static_assert(Check_tensor3d_kernel_2In_1Out<Kernel<std::int8_t>>::check_passed);
    static_assert(Check_tensor3d_kernel_2In_1Out<Kernel<std::uint8_t>>::check_passed);
    static_assert(Check_tensor3d_kernel_2In_1Out<Kernel<__half>>::check_passed);
    static_assert(Check_tensor3d_kernel_2In_1Out<Kernel<float>>::check_passed);
    static_assert(Check_tensor3d_kernel_2In_1Out<Kernel<double>>::check_passed);
    static constexpr bool check_passed = true;
};
