// glm_gradient_xyyhat.cuh -- Glm_gradient_xyyhat_spec / Glm_gradient_xyyhat_kernel<T>.
//
// Drop-in for the reference's kernel class of the same name
// (include/cuda/kernels/glm/glm_gradient_xyyhat.cuh:439-857 in gpu_algos):
// same spec members, command-line options, defaults and validation, same
// run_device_kernel / run_host_kernel signatures.  It computes the gradient of
//   L = sum_{t,task,obs} (Yhat - Y)^2 + lambda*(alpha*|M|_1 + (1-alpha)*|M|^2),
//   grad = 2 * sum_obs (Yhat - Y) X + lambda*(alpha*sign(M) + 2*(1-alpha)*M),
// with Yhat = X.M written to `temp` as the reference does.
//
// run_device_kernel makes one call into libglm_b200.so (glmb_gradient_<type>),
// which runs the fused single-pass sm_100a kernel (predict, residual and
// gradient in one read of X).  The reference's --gpu-algo values
// (fixed-grid, naive, warp, block) name thread-mapping variants of its two
// separate launches; they are all accepted and all run that one fused kernel.
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

struct Glm_gradient_xyyhat_spec {
    const std::string type_;
    const std::string gpu_algo_;
    const std::string cpu_algo_;
    const double lambda_;
    const double alpha_;
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
    // Y (ntargets, ntasks, nobs)
    const long n_cols_C_;
    const long n_rows_C_;
    const long n_sheets_C_;
    // grad_M (nfeatures, ntargets, ntasks)
    const long n_cols_D_;
    const long n_rows_D_;
    const long n_sheets_D_;
    // Yhat (ntargets, ntasks, nobs)
    const long n_cols_temp_;
    const long n_rows_temp_;
    const long n_sheets_temp_;

    // Informational: the fused kernel chooses its own launch shape.
    const dim3 fixed_grid_block_dim_;
    const long block_dim_;
    const dim3 grid_dim_;
    const size_t dynamic_shm_words_;

    constexpr static long DEFAULT_NOBS = 1000;
    constexpr static long DEFAULT_NTASKS = 10;
    constexpr static long DEFAULT_NTARGETS = 25;
    constexpr static long DEFAULT_NFEATURES = 25;
    constexpr static long DEFAULT_BLOCK_DIM = 8;
    constexpr static double DEFAULT_LAMBDA = 0.0;
    constexpr static double DEFAULT_ALPHA = 0.0;  // pure L2 regularisation
    constexpr static const char* DEFAULT_GPU_ALGO = "fused";

    static bool valid_gpu_algo(const std::string& a) {
        return a == "fused" || a == "fixed-grid" || a == "naive" || a == "warp" || a == "block";
    }
    static bool valid_type(const std::string& t) {
        return t == "half" || t == "single" || t == "float" || t == "double" || t == "int8" || t == "int16" ||
               t == "int32" || t == "int64" || t == "uint8" || t == "uint16" || t == "uint32" || t == "uint64";
    }

    inline static void add_kernel_spec_options(cxxopts::Options& options) {
        options.add_options()
            ("nfeatures,X", "Number of features", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NFEATURES)))
            ("ntargets,Y", "Number of targets", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NTARGETS)))
            ("ntasks,T", "Number of tasks", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NTASKS)))
            ("nobs,N", "Number of observations", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_NOBS)))
            ("lambda", "Regularization parameter", cxxopts::value<double>()->default_value(std::to_string(DEFAULT_LAMBDA)))
            ("alpha", "L1 mixing parameter (default to 0.0 for pure L2 regularization)",
             cxxopts::value<double>()->default_value(std::to_string(DEFAULT_ALPHA)))
            ("block-dim-x", "Number of threads in the x dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("block-dim-y", "Number of threads in the y dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("block-dim-z", "Number of threads in the z dimension per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("type", "Numeric type (half, single/float, double, int<n>, uint<n>)",
             cxxopts::value<std::string>()->default_value("float"))
            ("gpu-algo", "GPU algo to use (fused; fixed-grid, naive, warp, block are accepted and run fused)",
             cxxopts::value<std::string>()->default_value(DEFAULT_GPU_ALGO))
            ("cpu-algo", "CPU algo variant to benchmark against (nested-loop, matrix)",
             cxxopts::value<std::string>()->default_value("matrix"));
    }

    inline static Glm_gradient_xyyhat_spec make(const cxxopts::ParseResult& options_parsed) {
        const auto gpu_algo = options_parsed["gpu-algo"].as<std::string>();
        if (!valid_gpu_algo(gpu_algo)) {
            std::cerr << "[ERROR] --gpu-algo must be one of: fused, fixed-grid, naive, warp, block" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --gpu-algo: " + gpu_algo);
        }
        const auto cpu_algo = options_parsed["cpu-algo"].as<std::string>();
        if (cpu_algo != "nested-loop" && cpu_algo != "matrix") {
            std::cerr << "[ERROR] --cpu-algo must be one of: nested-loop, matrix" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --cpu-algo: " + cpu_algo);
        }
        const auto type = options_parsed["type"].as<std::string>();
        if (!valid_type(type)) {
            std::cerr << "[ERROR] --type must be one of: half, single/float, double, int<n>, uint<n>" << std::endl;
            throw cxxopts::exceptions::exception("Invalid --type: " + type);
        }
        const double lambda = options_parsed["lambda"].as<double>();
        const double alpha = options_parsed["alpha"].as<double>();
        if (lambda < 0 || alpha < 0 || alpha > 1)
            throw cxxopts::exceptions::exception("--lambda must be >= 0 and --alpha in [0, 1]");
        const long nf = options_parsed["nfeatures"].as<long>(), nt = options_parsed["ntargets"].as<long>();
        const long ntasks = options_parsed["ntasks"].as<long>(), nobs = options_parsed["nobs"].as<long>();
        if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0)
            throw cxxopts::exceptions::exception("sizes must be non-negative");
        const dim3 block{options_parsed["block-dim-x"].as<unsigned>(), options_parsed["block-dim-y"].as<unsigned>(),
                         options_parsed["block-dim-z"].as<unsigned>()};
        return Glm_gradient_xyyhat_spec(type, gpu_algo, cpu_algo, nf, nt, ntasks, nobs, lambda, alpha, block);
    }

    inline Glm_gradient_xyyhat_spec(const std::string& type, const std::string& gpu_algo,
                                    const std::string& cpu_algo, const long nfeatures, const long ntargets,
                                    const long ntasks, const long nobs, const double lambda, const double alpha,
                                    const dim3 fixed_grid_block_dim)
        : type_(type), gpu_algo_(gpu_algo), cpu_algo_(cpu_algo), lambda_(lambda), alpha_(alpha),
          nfeatures_(nfeatures), ntargets_(ntargets), ntasks_(ntasks), nobs_(nobs),
          niterations_(nobs * ntasks * ntargets),
          n_cols_A_(nfeatures), n_rows_A_(ntasks), n_sheets_A_(nobs),
          n_cols_B_(nfeatures), n_rows_B_(ntargets), n_sheets_B_(ntasks),
          n_cols_C_(ntargets), n_rows_C_(ntasks), n_sheets_C_(nobs),
          n_cols_D_(nfeatures), n_rows_D_(ntargets), n_sheets_D_(ntasks),
          n_cols_temp_(ntargets), n_rows_temp_(ntasks), n_sheets_temp_(nobs),
          fixed_grid_block_dim_(fixed_grid_block_dim),
          block_dim_(long(fixed_grid_block_dim.x) * fixed_grid_block_dim.y * fixed_grid_block_dim.z),
          grid_dim_(1, 1, 1),
          dynamic_shm_words_(0) {}
};

static_assert(Check_tensor3d_kernel_spec_3In_1Out<Glm_gradient_xyyhat_spec>::check_passed);

template <CUDA_scalar Number_>
class Glm_gradient_xyyhat_kernel {
   public:
    using Number = Number_;
    using Kernel_spec = Glm_gradient_xyyhat_spec;

    const Kernel_spec spec_;

    explicit Glm_gradient_xyyhat_kernel(const Kernel_spec spec) : spec_(spec) {}

    void run_device_kernel(const Number* const gpu_data_X, const Number* const gpu_data_M,
                           const Number* const gpu_data_Y, Number* const gpu_data_grad_M,
                           Number* const gpu_data_Yhat, cudaStream_t stream) {
        const uint32_t flags = GLMB_GRAD_REGULARIZE | (gpu_data_Yhat != nullptr ? GLMB_GRAD_WRITE_YHAT : 0u);
        const int st = glm_host::abi_gradient(gpu_data_X, gpu_data_M, gpu_data_Y, gpu_data_grad_M, gpu_data_Yhat,
                                              spec_.nfeatures_, spec_.ntargets_, spec_.ntasks_, spec_.nobs_,
                                              spec_.lambda_, spec_.alpha_, flags, stream);
        std::cout << "[INFO] glmb_gradient_" << glm_host::abi_suffix(gpu_data_X) << "(nfeatures="
                  << spec_.nfeatures_ << ", ntargets=" << spec_.ntargets_ << ", ntasks=" << spec_.ntasks_
                  << ", nobs=" << spec_.nobs_ << ", lambda=" << spec_.lambda_ << ", alpha=" << spec_.alpha_
                  << ") path=" << glmb_last_path() << std::endl;
        cuda_check_error(st, "glmb_gradient");
    }

    Tensor3D<Number> run_host_kernel(const Tensor3D<Number>& X, const Tensor3D<Number>& M,
                                     const Tensor3D<Number>& Y) {
        return glm_host::gradient(X, M, Y, spec_.lambda_, spec_.alpha_, true, spec_.cpu_algo_ == "matrix");
    }
};

static_assert(Check_tensor3d_kernel_3In_1Out_template<Glm_gradient_xyyhat_kernel>::check_passed);
