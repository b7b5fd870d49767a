// cuda/kernel_api/tensor3d_3in_1out.cuh -- compile-time contract of a
// kernel with three Tensor3D inputs (A, B, C), one output D and a temp.
//
// Same requirements as the reference's TENSOR3D_KERNEL_SPEC_3IN_1OUT /
// TENSOR3D_KERNEL_3IN_1OUT (include/cuda/kernel_api/tensor3d_3in_1out.cuh:32-149
// in gpu_algos): the spec exposes the fifteen `const long n_{cols,rows,sheets}_X_`
// extents and dim3-convertible block/grid sizes; the kernel exposes `spec_`,
// `run_device_kernel(const A*, const B*, const C*, D*, Temp*, cudaStream_t)`
// and `run_host_kernel(const Tensor3D<A>&, const Tensor3D<B>&, const Tensor3D<C>&)`
// returning the output tensor; a kernel template must satisfy this for
// int8, uint8, __half, float and double.
#pragma once

#include <concepts>
#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#include "common/types/tensor3d.hpp"
#include "cuda/kernel_detect_types.cuh"
#include "cuda/type_traits.cuh"

template <typename S>
concept TENSOR3D_KERNEL_SPEC_3IN_1OUT = requires(S spec) {
    { spec.n_rows_A_ } -> std::same_as<const long&>;
    { spec.n_cols_A_ } -> std::same_as<const long&>;
    { spec.n_sheets_A_ } -> std::same_as<const long&>;
    { spec.n_rows_B_ } -> std::same_as<const long&>;
    { spec.n_cols_B_ } -> std::same_as<const long&>;
    { spec.n_sheets_B_ } -> std::same_as<const long&>;
    { spec.n_rows_C_ } -> std::same_as<const long&>;
    { spec.n_cols_C_ } -> std::same_as<const long&>;
    { spec.n_sheets_C_ } -> std::same_as<const long&>;
    { spec.n_rows_D_ } -> std::same_as<const long&>;
    { spec.n_cols_D_ } -> std::same_as<const long&>;
    { spec.n_sheets_D_ } -> std::same_as<const long&>;
    { spec.n_rows_temp_ } -> std::same_as<const long&>;
    { spec.n_cols_temp_ } -> std::same_as<const long&>;
    { spec.n_sheets_temp_ } -> std::same_as<const long&>;
    { dim3(spec.block_dim_) } -> std::same_as<dim3>;
    { dim3(spec.grid_dim_) } -> std::same_as<dim3>;
};

template <typename S>
struct Check_tensor3d_kernel_spec_3In_1Out {
    static_assert(TENSOR3D_KERNEL_SPEC_3IN_1OUT<S>, "not a valid TENSOR3D_KERNEL_SPEC_3IN_1OUT");
    static constexpr bool check_passed = true;
};

template <typename K>
concept TENSOR3D_KERNEL_3IN_1OUT = requires(K kernel) {
    typename K::Number;
    typename K::Kernel_spec;
    requires TENSOR3D_KERNEL_SPEC_3IN_1OUT<typename K::Kernel_spec>;
    { kernel.spec_ } -> std::same_as<const typename K::Kernel_spec&>;
    { kernel.run_device_kernel(std::declval<const typename detect::Numbers<K>::A*>(),
                               std::declval<const typename detect::Numbers<K>::B*>(),
                               std::declval<const typename detect::Numbers<K>::C*>(),
                               std::declval<typename detect::Numbers<K>::D*>(),
                               std::declval<typename detect::Numbers<K>::Temp*>(),
                               std::declval<cudaStream_t>()) } -> std::same_as<void>;
    { kernel.run_host_kernel(std::declval<const Tensor3D<typename detect::Numbers<K>::A>&>(),
                             std::declval<const Tensor3D<typename detect::Numbers<K>::B>&>(),
                             std::declval<const Tensor3D<typename detect::Numbers<K>::C>&>()) }
        -> std::same_as<Tensor3D<typename detect::Numbers<K>::D>>;
};

template <typename K>
struct Check_tensor3d_kernel_3In_1Out {
    static_assert(TENSOR3D_KERNEL_3IN_1OUT<K>, "not a valid TENSOR3D_KERNEL_3IN_1OUT");
    static constexpr bool check_passed = true;
};

template <template <CUDA_scalar> class Kernel>
struct Check_tensor3d_kernel_3In_1Out_template {
    static_assert(Check_tensor3d_kernel_3In_1Out<Kernel<std::int8_t>>::check_passed);
    static_assert(Check_tensor3d_kernel_3In_1Out<Kernel<std::uint8_t>>::check_passed);
    static_assert(Check_tensor3d_kernel_3In_1Out<Kernel<__half>>::check_passed);
    static_assert(Check_tensor3d_kernel_3In_1Out<Kernel<float>>::check_passed);
    static_assert(Check_tensor3d_kernel_3In_1Out<Kernel<double>>::check_passed);
    static constexpr bool check_passed = true;
};
