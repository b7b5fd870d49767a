// host_api_probe.cpp -- exposes pieces of the C++ host mirror (Tensor3D, the
// option parser, the seeded initialisation, the kernel classes' host
// computations) through extern "C" so the CPU tests can drive them with
// ctypes.  Test code only; built by tests/test_host_api.py.
#include <cstdint>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include "common/benchmark_options.hpp"
#include "common/types/tensor3d.hpp"
#include "cuda/kernels/glm/glm_gradient_naive.cuh"
#include "cuda/kernels/glm/glm_gradient_xyyhat.cuh"
#include "cuda/kernels/glm/glm_loss_myyhat.cuh"
#include "cuda/kernels/glm/glm_predict_naive.cuh"
#include "cxxopts.hpp"

namespace {

template <typename T>
Tensor3D<T> make(const T* data, long cols, long rows, long sheets) {
    Tensor3D<T> t(cols, rows, sheets);
    if (t.vector_.size()) std::memcpy(t.data(), data, t.vector_.size() * sizeof(T));
    return t;
}

template <typename T>
void host_gradient(const T* X, const T* M, const T* Y, T* grad, long nf, long nt, long ntasks, long nobs,
                   double lambda, double alpha, int reg, int matrix) {
    const auto tx = make(X, nf, ntasks, nobs), tm = make(M, nf, nt, ntasks), ty = make(Y, nt, ntasks, nobs);
    Tensor3D<T> g = [&] {
        if (reg) {
            Glm_gradient_xyyhat_kernel<T> k(Glm_gradient_xyyhat_spec("float", "fused", matrix ? "matrix" : "nested-loop",
                                                                     nf, nt, ntasks, nobs, lambda, alpha, dim3(8, 8, 8)));
            return k.run_host_kernel(tx, tm, ty);
        }
        Glm_gradient_naive_kernel<T> k(Glm_gradient_naive_spec("float", matrix ? "matrix" : "nested-loop", nf, nt,
                                                               ntasks, nobs, dim3(8, 8, 8), false));
        return k.run_host_kernel(tx, tm, ty);
    }();
    std::memcpy(grad, g.data(), g.vector_.size() * sizeof(T));
}

template <typename T>
void host_predict(const T* X, const T* M, T* Yhat, long nf, long nt, long ntasks, long nobs) {
    Glm_predict_naive_kernel<T> k(Glm_predict_naive_spec("float", "fused", nf, nt, ntasks, nobs, dim3(32, 4, 4)));
    const Tensor3D<T> y = k.run_host_kernel(make(X, nf, ntasks, nobs), make(M, nf, nt, ntasks));
    std::memcpy(Yhat, y.data(), y.vector_.size() * sizeof(T));
}

template <typename T>
void host_loss(const T* M, const T* Y, const T* Yhat, T* loss, long nf, long nt, long ntasks, long nobs,
               double lambda, double alpha) {
    Glm_loss_myyhat_kernel<T> k(Glm_loss_myyhat_spec("float", nf, nt, ntasks, nobs, lambda, alpha, 512));
    const Tensor3D<T> l = k.run_host_kernel(make(M, nf, nt, ntasks), make(Y, nt, ntasks, nobs),
                                            make(Yhat, nt, ntasks, nobs));
    loss[0] = l.data()[0];
}

std::string g_text;

}  // namespace

extern "C" {

#define PROBE(SFX, T)                                                                                     \
    void probe_gradient_##SFX(const T* X, const T* M, const T* Y, T* g, long nf, long nt, long ntasks,   \
                              long nobs, double lambda, double alpha, int reg, int matrix) {              \
        host_gradient<T>(X, M, Y, g, nf, nt, ntasks, nobs, lambda, alpha, reg, matrix);                   \
    }                                                                                                     \
    void probe_predict_##SFX(const T* X, const T* M, T* Yh, long nf, long nt, long ntasks, long nobs) {  \
        host_predict<T>(X, M, Yh, nf, nt, ntasks, nobs);                                                  \
    }                                                                                                     \
    void probe_loss_##SFX(const T* M, const T* Y, const T* Yh, T* loss, long nf, long nt, long ntasks,   \
                          long nobs, double lambda, double alpha) {                                       \
        host_loss<T>(M, Y, Yh, loss, nf, nt, ntasks, nobs, lambda, alpha);                                \
    }                                                                                                     \
    void probe_randomize_##SFX(T* out, long n, long seed) {                                               \
        Tensor3D<T> t(n, 1, 1);                                                                           \
        t.randomize(seed);                                                                                \
        std::memcpy(out, t.data(), n * sizeof(T));                                                        \
    }

PROBE(f32, float)
PROBE(f64, double)
PROBE(i32, int32_t)
PROBE(u8, uint8_t)
PROBE(i64, int64_t)

// Parses argv with the GLM xyyhat options; returns 0 and a "key=value;..."
// summary, or 1 and the exception text.
int probe_parse(int argc, const char** argv, const char** out) {
    cxxopts::Options options("probe", "option parser probe");
    add_benchmark_options(options);
    Glm_gradient_xyyhat_spec::add_kernel_spec_options(options);
    try {
        const auto r = options.parse(argc, argv);
        const auto spec = Glm_gradient_xyyhat_spec::make(r);
        std::ostringstream os;
        os << "nfeatures=" << spec.nfeatures_ << ";ntargets=" << spec.ntargets_ << ";ntasks=" << spec.ntasks_
           << ";nobs=" << spec.nobs_ << ";lambda=" << spec.lambda_ << ";alpha=" << spec.alpha_
           << ";type=" << spec.type_ << ";gpu_algo=" << spec.gpu_algo_ << ";cpu_algo=" << spec.cpu_algo_
           << ";seed=" << r["seed"].as<long>() << ";verbose=" << r["verbose"].as<bool>()
           << ";force=" << r["force"].as<bool>() << ";help=" << r.count("help")
           << ";init=" << r["init-method"].as<std::string>() << ";bx=" << spec.fixed_grid_block_dim_.x;
        g_text = os.str();
        *out = g_text.c_str();
        return 0;
    } catch (const cxxopts::exceptions::exception& e) {
        g_text = e.what();
        *out = g_text.c_str();
        return 1;
    }
}

}  // extern "C"
