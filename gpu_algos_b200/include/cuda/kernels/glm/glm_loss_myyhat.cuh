// glm_loss_myyhat.cuh -- Glm_loss_myyhat_spec / Glm_loss_myyhat_kernel<T>.
//
// Drop-in for the reference's kernel class of the same name
// (include/cuda/kernels/glm/glm_loss_myyhat.cuh:161-402 in gpu_algos): the
// objective
//   loss = sum_{t,task,obs} (Yhat - Y)^2 + lambda*(alpha*|M|_1 + (1-alpha)*|M|^2)
// from the model M, the responses Y and the predictions Yhat, as a 1 x 1 x 1
// tensor.  Same options, defaults and validation; run_device_kernel makes one
// call into libglm_b200.so (glmb_loss_<type>, a streaming reduction over Y
// and Yhat plus one pass over M).
//
// One deliberate difference: the reference's spec gives its A and B tensors
// the shapes of X (nfeatures, ntasks, nobs) and M (nfeatures, ntargets,
// ntasks) although the kernel reads them as M and Y (it reads Y past the end
// of B whenever nobs > nfeatures); here A has M's shape and B has Y's, which
// is what the kernel reads.
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

struct Glm_loss_myyhat_spec {
    const std::string type_;
    const double lambda_;
    const double alpha_;
    const long nfeatures_;
    const long ntargets_;
    const long ntasks_;
    const long nobs_;
    const long niterations_;

    // M (nfeatures, ntargets, ntasks)
    const long n_cols_A_;
    const long n_rows_A_;
    const long n_sheets_A_;
    // Y (ntargets, ntasks, nobs)
    const long n_cols_B_;
    const long n_rows_B_;
    const long n_sheets_B_;
    // Yhat (ntargets, ntasks, nobs)
    const long n_cols_C_;
    const long n_rows_C_;
    const long n_sheets_C_;
    // loss (1, 1, 1)
    const long n_cols_D_;
    const long n_rows_D_;
    const long n_sheets_D_;
    // temp: unused (the library keeps its per-CTA partials in its own scratch)
    const long n_cols_temp_;
    const long n_rows_temp_;
    const long n_sheets_temp_;

    const long size_Y_;
    const long size_M_;
    // Informational: the reduction chooses its own launch shape.
    const long block_dim_;
    const dim3 grid_dim_;
    const size_t dynamic_shm_words_;

    constexpr static long DEFAULT_NOBS = 1000;
    constexpr static long DEFAULT_NTASKS = 10;
    constexpr static long DEFAULT_NTARGETS = 25;
    constexpr static long DEFAULT_NFEATURES = 25;
    constexpr static long DEFAULT_BLOCK_DIM = 512;
    constexpr static double DEFAULT_LAMBDA = 0.0;
    constexpr static double DEFAULT_ALPHA = 0.0;  // pure L2 regularisation

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
            ("block-dim", "Number of threads per block",
             cxxopts::value<unsigned>()->default_value(std::to_string(DEFAULT_BLOCK_DIM)))
            ("type", "Numeric type (half, single/float, double, int<n>, uint<n>)",
             cxxopts::value<std::string>()->default_value("float"));
    }

    inline static Glm_loss_myyhat_spec make(const cxxopts::ParseResult& options_parsed) {
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
        return Glm_loss_myyhat_spec(type, nf, nt, ntasks, nobs, lambda, alpha,
                                    options_parsed["block-dim"].as<unsigned>());
    }

    inline Glm_loss_myyhat_spec(const std::string& type, const long nfeatures, const long ntargets,
                                const long ntasks, const long nobs, const double lambda, const double alpha,
                                const unsigned block_dim)
        : type_(type), lambda_(lambda), alpha_(alpha), nfeatures_(nfeatures), ntargets_(ntargets),
          ntasks_(ntasks), nobs_(nobs), niterations_(nobs * ntasks * ntargets),
          n_cols_A_(nfeatures), n_rows_A_(ntargets), n_sheets_A_(ntasks),
          n_cols_B_(ntargets), n_rows_B_(ntasks), n_sheets_B_(nobs),
          n_cols_C_(ntargets), n_rows_C_(ntasks), n_sheets_C_(nobs),
          n_cols_D_(1), n_rows_D_(1), n_sheets_D_(1),
          n_cols_temp_(0), n_rows_temp_(0), n_sheets_temp_(0),
          size_Y_(ntargets * ntasks * nobs), size_M_(nfeatures * ntargets * ntasks),
          block_dim_(block_dim), grid_dim_(1, 1, 1), dynamic_shm_words_(0) {}
};

static_assert(Check_tensor3d_kernel_spec_3In_1Out<Glm_loss_myyhat_spec>::check_passed);

template <CUDA_scalar Number_>
class Glm_loss_myyhat_kernel {
   public:
    using Number = Number_;
    using Kernel_spec = Glm_loss_myyhat_spec;

    const Kernel_spec spec_;

    explicit Glm_loss_myyhat_kernel(const Kernel_spec spec) : spec_(spec) {}

    void run_device_kernel(const Number* const gpu_data_M, const Number* const gpu_data_Y,
                           const Number* const gpu_data_Yhat, Number* const gpu_data_loss,
                           Number* const /*gpu_data_temp (unused)*/, cudaStream_t stream) {
        const int st = glm_host::abi_loss(gpu_data_M, gpu_data_Y, gpu_data_Yhat, gpu_data_loss, spec_.nfeatures_,
                                          spec_.ntargets_, spec_.ntasks_, spec_.nobs_, spec_.lambda_,
                                          spec_.alpha_, stream);
        std::cout << "[INFO] glmb_loss_" << glm_host::abi_suffix(gpu_data_M) << "(nfeatures=" << spec_.nfeatures_
                  << ", ntargets=" << spec_.ntargets_ << ", ntasks=" << spec_.ntasks_ << ", nobs=" << spec_.nobs_
                  << ", lambda=" << spec_.lambda_ << ", alpha=" << spec_.alpha_ << ")" << std::endl;
        cuda_check_error(st, "glmb_loss");
    }

    Tensor3D<Number> run_host_kernel(const Tensor3D<Number>& M, const Tensor3D<Number>& Y,
                                     const Tensor3D<Number>& Yhat) {
        return glm_host::loss(M, Y, Yhat, spec_.lambda_, spec_.alpha_);
    }
};

static_assert(Check_tensor3d_kernel_3In_1Out_template<Glm_loss_myyhat_kernel>::check_passed);
