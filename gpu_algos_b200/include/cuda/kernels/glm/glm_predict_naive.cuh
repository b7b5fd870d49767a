// glm_predict_naive.cuh -- Glm_predict_naive_spec / Glm_predict_naive_kernel<T>.
//
// Drop-in for the reference's kernel class of the same name
// (include/cuda/kernels/glm/glm_predict_naive.cuh:369-648 in gpu_algos):
//   Yhat[target, task, obs] = sum_feature M[feature, target, task] * X[feature, task, obs].
// run_device_kernel makes one call into libglm_b200.so (glmb_predict_<type>).
// The reference's --gpu-algo values (fixed-grid, naive, warp, group, block)
// are accepted; all run the same coalesced warp-per-row sm_100a kernel.
#pragma once

#include <iostream>
#include <string>

#include <cuda_runtime.h>

#include "common/types/tensor3d.hpp"
#include "cuda/check_errors.cuh"
#include "cuda/kernel_api/tensor3d_2in_1out.cuh"
#include "cuda/kernels/glm/glm_host.hpp"
#include "cuda/type_traits.cuh"
#include "cxxopts.hpp"

struct Glm_predict_naive_spec {
    const std::string type_;
    const std::string gpu_algo_;
    const long nfeatures_;
    const long ntargets_;
    const long ntasks_;
    const long nobs_;
    const long niterations_;

    // X (nfeatures, ntasks, nobs)
    const long n_cols_A_;
    const long n_rows_A_;
    const long n_sheets_A_;
    // M (nfeatures, ntargets, ntasks)
    const long n_cols_B_;
    const long n_rows_B_;
    const long n_sheets_B_;
    // Yhat (ntargets, ntasks, nobs)
    const long n_cols_C_;
    const long n_rows_C_;
    const long n_sheets_C_;
    // temp: unused
    const long n_cols_temp_;
    const long n_rows_temp_;
    const long n_sheets_temp_;

    const dim3 fixed_grid_block_dim_;
    const long block_dim_;
    const dim3 grid_dim_;
    const size_t dynamic_shared_mem_words_;

    constexpr static long DEFAULT_NOBS = 1000;
    constexpr static long DEFAULT_NTASKS = 10;
    constexpr static long DEFAULT_NTARGETS = 25;
    constexpr static long DEFAULT_NFEATURES = 25;
    constexpr static long DEFAULT_BLOCK_DIM_X = 32;
    constexpr static long DEFAULT_BLOCK_DIM_Y = 4;
    constexpr static long DEFAULT_BLOCK_DIM_Z = 4;
    constexpr static const char* DEFAULT_GPU_ALGO = "fused";

    inline static void add_kernel_spec_options(cxxopts::Options& options) {
        options.add_options()
            ("nfeatures,X", "Number of features", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NFEATURES)))
            ("ntargets,Y", "Number of targets", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NTARGETS)))
            ("ntasks,T", "Number of tasks", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NTASKS)))
            ("nobs,N", "Number of observations", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NOBS)))
            ("block-dim-x", "Number of threads in the x dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM_X)))
            ("block-dim-y", "Number of threads in the y dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM_Y)))
            ("block-dim-z", "Number of threads in the z dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM_Z)))
            ("gpu-algo", "GPU algo to use (fused; fixed-grid, naive, warp, group, block are accepted and run fused)",
             cxxopts::value<std::string>()->default_value(DEFAULT_GPU_ALGO))
            ("type", "Numeric type (half, single/float, double, int<n>, uint<n>)",
             cxxopts::value<std::string>()->default_value("float"));
    }

    inline static Glm_predict_naive_spec make(const cxxopts::ParseResult& options_parsed) {
        const auto gpu_algo = options_parsed["gpu-algo"].as<std::string>();
        if (gpu_algo != "fused" && gpu_algo != "fixed-grid" && gpu_algo != "naive" && gpu_algo != "group" &&
            gpu_algo != "warp" && gpu_algo != "block") {
            std::cerr << "[ERROR] --gpu-algo must be one of: fused, fixed-grid, naive, warp, group, block" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --gpu-algo: " + gpu_algo);
        }
        const auto type = options_parsed["type"].as<std::string>();
        if (type != "half" && type != "single" && type != "float" && type != "double" && type != "int8" &&
            type != "int16" && type != "int32" && type != "int64" && type != "uint8" && type != "uint16" &&
            type != "uint32" && type != "uint64") {
            std::cerr << "[ERROR] --type must be one of: half, single/float, double, int<n>, uint<n>" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --type: " + type);
        }
        const long nf = options_parsed["nfeatures"].as<long>(), nt = options_parsed["ntargets"].as<long>();
        const long ntasks = options_parsed["ntasks"].as<long>(), nobs = options_parsed["nobs"].as<long>();
        if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0)
            throw cxxopts::exceptions::exception("sizes must be non-negative");
        const dim3 block{options_parsed["block-dim-x"].as<unsigned>(), options_parsed["block-dim-y"].as<unsigned>(),
                         options_parsed["block-dim-z"].as<unsigned>()};
        return Glm_predict_naive_spec(type, gpu_algo, nf, nt, ntasks, nobs, block);
    }

    Glm_predict_naive_spec(const std::string& type, const std::string& gpu_algo, const long nfeatures,
                           const long ntargets, const long ntasks, const long nobs, const dim3 fixed_grid_block_dim)
        : type_(type), gpu_algo_(gpu_algo), nfeatures_(nfeatures), ntargets_(ntargets), ntasks_(ntasks),
          nobs_(nobs), niterations_(nobs * ntasks * ntargets),
          n_cols_A_(nfeatures), n_rows_A_(ntasks), n_sheets_A_(nobs),
          n_cols_B_(nfeatures), n_rows_B_(ntargets), n_sheets_B_(ntasks),
          n_cols_C_(ntargets), n_rows_C_(ntasks), n_sheets_C_(nobs),
          n_cols_temp_(0), n_rows_temp_(0), n_sheets_temp_(0),
          fixed_grid_block_dim_(fixed_grid_block_dim),
          block_dim_(long(fixed_grid_block_dim.x) * fixed_grid_block_dim.y * fixed_grid_block_dim.z),
          grid_dim_(1, 1, 1), dynamic_shared_mem_words_(0) {}
};

static_assert(Check_tensor3d_kernel_spec_2In_1Out<Glm_predict_naive_spec>::check_passed);

template <CUDA_scalar Number_>
class Glm_predict_naive_kernel {
   public:
    using Number = Number_;
    using Kernel_spec = Glm_predict_naive_spec;

    const Kernel_spec spec_;

    explicit Glm_predict_naive_kernel(const Kernel_spec spec) : spec_(spec) {}

    void run_device_kernel(const Number* const gpu_data_X, const Number* const gpu_data_M,
                           Number* const gpu_data_Yhat, Number* const /*gpu_data_temp (unused)*/,
                           cudaStream_t stream) {
        const int st = glm_host::abi_predict(gpu_data_X, gpu_data_M, gpu_data_Yhat, spec_.nfeatures_,
                                             spec_.ntargets_, spec_.ntasks_, spec_.nobs_, stream);
        std::cout << "[INFO] glmb_predict_" << glm_host::abi_suffix(gpu_data_X) << "(nfeatures=" << spec_.nfeatures_
                  << ", ntargets=" << spec_.ntargets_ << ", ntasks=" << spec_.ntasks_ << ", nobs=" << spec_.nobs_
                  << ") path=" << glmb_last_path() << std::endl;
        cuda_check_error(st, "glmb_predict");
    }

    Tensor3D<Number> run_host_kernel(const Tensor3D<Number>& X, const Tensor3D<Number>& M) {
        return glm_host::predict(X, M);
    }
};

static_assert(Check_tensor3d_kernel_2In_1Out_template<Glm_predict_naive_kernel>::check_passed);
