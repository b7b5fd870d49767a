// glm_gradient_naive.cuh -- Glm_gradient_naive_spec / Glm_gradient_naive_kernel<T>.
//
// Drop-in for the reference's kernel class of the same name
// (include/cuda/kernels/glm/glm_gradient_naive.cuh:178-461 in gpu_algos): the
// unregularised gradient grad = 2 * sum_obs (X.M - Y) X, no temp tensor.
// run_device_kernel makes one call into libglm_b200.so (glmb_gradient_<type>
// without GLMB_GRAD_REGULARIZE).  --optimize-launch is accepted; the fused
// kernel always sizes its own grid from the SM count and occupancy.
#pragma once

#include <iostream>
#include <string>

#include <cuda_runtime.h>

#include "common/types/tensor3d.hpp"
#include "cuda/check_errors.cuh"
#include "cuda/kernel_api/tensor3d_3in_1out.cuh"
#include "cuda/kernels/glm/glm_host.hpp"
#include "cuda/type_traits.cuh"
#include "cxxopts.hpp"

struct Glm_gradient_naive_spec {
    const std::string type_;
    const std::string cpu_algo_;
    const long nfeatures_;
    const long ntargets_;
    const long ntasks_;
    const long nobs_;

    const long n_cols_A_;
    const long n_rows_A_;
    const long n_sheets_A_;
    const long n_cols_B_;
    const long n_rows_B_;
    const long n_sheets_B_;
    const long n_cols_C_;
    const long n_rows_C_;
    const long n_sheets_C_;
    const long n_cols_D_;
    const long n_rows_D_;
    const long n_sheets_D_;
    // temp: unused
    const long n_cols_temp_;
    const long n_rows_temp_;
    const long n_sheets_temp_;

    const dim3 block_dim_;
    const dim3 grid_dim_;
    const size_t dynamic_shared_mem_words_ = 0;
    const bool optimize_launch_;

    constexpr static long DEFAULT_NOBS = 1000;
    constexpr static long DEFAULT_NTASKS = 10;
    constexpr static long DEFAULT_NTARGETS = 25;
    constexpr static long DEFAULT_NFEATURES = 25;
    constexpr static long DEFAULT_BLOCK_DIM = 8;

    inline static void add_kernel_spec_options(cxxopts::Options& options) {
        options.add_options()
            ("nfeatures,X", "Number of features", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NFEATURES)))
            ("ntargets,Y", "Number of targets", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NTARGETS)))
            ("ntasks,T", "Number of tasks", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NTASKS)))
            ("nobs,N", "Number of observations", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NOBS)))
            ("block-dim-x", "Number of threads in the x dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("block-dim-y", "Number of threads in the y dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("block-dim-z", "Number of threads in the z dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("optimize-launch", "Use occupancy API to determine optimal launch configuration")
            ("type", "Numeric type (half, single/float, double, int<n>, uint<n>)",
             cxxopts::value<std::string>()->default_value("float"))
            ("cpu-algo", "CPU algo variant to benchmark against (nested-loop, matrix)",
             cxxopts::value<std::string>()->default_value("matrix"));
    }

    inline static Glm_gradient_naive_spec make(const cxxopts::ParseResult& options_parsed) {
        const auto type = options_parsed["type"].as<std::string>();
        if (type != "half" && type != "single" && type != "float" && type != "double" && type != "int8" &&
            type != "int16" && type != "int32" && type != "int64" && type != "uint8" && type != "uint16" &&
            type != "uint32" && type != "uint64") {
            std::cerr << "[ERROR] --type must be one of: half, single/float, double, int<n>, uint<n>" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --type: " + type);
        }
        const auto cpu_algo = options_parsed["cpu-algo"].as<std::string>();
        if (cpu_algo != "nested-loop" && cpu_algo != "matrix") {
            std::cerr << "[ERROR] --cpu-algo must be one of: nested-loop, matrix" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --cpu-algo: " + cpu_algo);
        }
        const long nf = options_parsed["nfeatures"].as<long>(), nt = options_parsed["ntargets"].as<long>();
        const long ntasks = options_parsed["ntasks"].as<long>(), nobs = options_parsed["nobs"].as<long>();
        if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0)
            throw cxxopts::exceptions::exception("sizes must be non-negative");
        const dim3 block{options_parsed["block-dim-x"].as<unsigned>(), options_parsed["block-dim-y"].as<unsigned>(),
                         options_parsed["block-dim-z"].as<unsigned>()};
        return Glm_gradient_naive_spec(type, cpu_algo, nf, nt, ntasks, nobs, block,
                                       options_parsed.count("optimize-launch") > 0);
    }

    inline Glm_gradient_naive_spec(const std::string& type, const std::string& cpu_algo, const long nfeatures,
                                   const long ntargets, const long ntasks, const long nobs, const dim3 block_dim,
                                   const bool optimize_launch)
        : type_(type), cpu_algo_(cpu_algo), nfeatures_(nfeatures), ntargets_(ntargets), ntasks_(ntasks),
          nobs_(nobs),
          n_cols_A_(nfeatures), n_rows_A_(ntasks), n_sheets_A_(nobs),
          n_cols_B_(nfeatures), n_rows_B_(ntargets), n_sheets_B_(ntasks),
          n_cols_C_(ntargets), n_rows_C_(ntasks), n_sheets_C_(nobs),
          n_cols_D_(nfeatures), n_rows_D_(ntargets), n_sheets_D_(ntasks),
          n_cols_temp_(0), n_rows_temp_(0), n_sheets_temp_(0),
          block_dim_(block_dim), grid_dim_(1, 1, 1), optimize_launch_(optimize_launch) {}
};

static_assert(Check_tensor3d_kernel_spec_3In_1Out<Glm_gradient_naive_spec>::check_passed);

template <CUDA_scalar Number_>
class Glm_gradient_naive_kernel {
   public:
    using Number = Number_;
    using Kernel_spec = Glm_gradient_naive_spec;

    const Kernel_spec spec_;

    explicit Glm_gradient_naive_kernel(const Kernel_spec spec) : spec_(spec) {}

    void run_device_kernel(const Number* const gpu_data_X, const Number* const gpu_data_M,
                           const Number* const gpu_data_Y, Number* const gpu_data_grad_M,
                           Number* const /*gpu_data_temp (unused)*/, cudaStream_t stream) {
        const int st = glm_host::abi_gradient(gpu_data_X, gpu_data_M, gpu_data_Y, gpu_data_grad_M, nullptr,
                                              spec_.nfeatures_, spec_.ntargets_, spec_.ntasks_, spec_.nobs_, 0.0,
                                              0.0, 0u, stream);
        std::cout << "[INFO] glmb_gradient_" << glm_host::abi_suffix(gpu_data_X) << "(nfeatures="
                  << spec_.nfeatures_ << ", ntargets=" << spec_.ntargets_ << ", ntasks=" << spec_.ntasks_
                  << ", nobs=" << spec_.nobs_ << ", unregularised) path=" << glmb_last_path() << std::endl;
        cuda_check_error(st, "glmb_gradient");
    }

    Tensor3D<Number> run_host_kernel(const Tensor3D<Number>& X, const Tensor3D<Number>& M,
                                     const Tensor3D<Number>& Y) {
        return glm_host::gradient(X, M, Y, 0.0, 0.0, false, spec_.cpu_algo_ == "matrix");
    }
};

static_assert(Check_tensor3d_kernel_3In_1Out_template<Glm_gradient_naive_kernel>::check_passed);
