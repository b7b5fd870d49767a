// glm_host.hpp -- host (CPU) GLM arithmetic behind the kernel classes'
// run_host_kernel, and the typed bridge from the kernel classes to the C ABI.
//
// run_host_kernel is the reference API's CPU implementation (the driver
// compares the GPU result with it).  Results are rounded to the Number type
// as the reference's are; sums are carried wider than the reference's own
// Eigen product so that the driver's check (relative error <= 2^-20 for
// float) measures the GPU's rounding rather than the host's: float in
// double, double in long double, half in float.  Integers compute modulo
// 2^bits (in the unsigned type of 32 or 64 bits, so wrapping is defined),
// bit-identical to the reference.
#pragma once

#include <algorithm>
#include <cstdint>
#include <type_traits>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common/types/tensor3d.hpp"
#include "cuda/type_traits.cuh"
#include "glm_b200.h"

namespace glm_host {

template <typename T>
struct Arith {
    using type = std::conditional_t<
        std::is_same_v<T, __half>, float,
        std::conditional_t<std::is_same_v<T, float>, double,
                           std::conditional_t<std::is_same_v<T, double>, long double,
                                              std::conditional_t<(sizeof(T) <= 4), uint32_t, uint64_t>>>>;
};
template <typename T>
using arith_t = typename Arith<T>::type;

template <typename T>
inline arith_t<T> up(T v) {
    if constexpr (std::is_same_v<T, __half>) return __half2float(v);
    else return static_cast<arith_t<T>>(v);
}
template <typename T>
inline T down(arith_t<T> v) {
    if constexpr (std::is_same_v<T, __half>) return __float2half_rn(v);
    else return static_cast<T>(v);
}
template <typename T>
inline T from_double(double d) {
    if constexpr (std::is_same_v<T, __half>) return __double2half(d);
    else return static_cast<T>(d);
}
template <typename T>
inline int sign_of(T v) {
    return is_positive(v) ? 1 : (is_negative(v) ? -1 : 0);
}

// Yhat(t, task, obs) = sum_f M(f, t, task) * X(f, task, obs)
// (glm_predict_naive.cuh:631-647 in gpu_algos).
template <typename T>
Tensor3D<T> predict(const Tensor3D<T>& X, const Tensor3D<T>& M) {
    const long nf = X.cols(), ntasks = X.rows(), nobs = X.sheets(), nt = M.rows();
    Tensor3D<T> Yhat(nt, ntasks, nobs);
#pragma omp parallel for schedule(static)
    for (long obs = 0; obs < nobs; ++obs)
        for (long task = 0; task < ntasks; ++task)
            for (long t = 0; t < nt; ++t) {
                const T* x = &X(0, task, obs);
                const T* m = &M(0, t, task);
                arith_t<T> s = 0;
                for (long f = 0; f < nf; ++f) s += up(m[f]) * up(x[f]);
                Yhat(t, task, obs) = down<T>(s);
            }
    return Yhat;
}

// grad(f, t, task) = 2 * sum_obs (Yhat - Y)(t, task, obs) * X(f, task, obs)
// [+ lambda*(alpha*sign(M) + 2*(1-alpha)*M)], the per-task product
// 2*(M X^T - Y^T) X of glm_gradient_xyyhat.cuh:813-852 in gpu_algos.
// `panel` observations are summed sequentially before being added into the
// result (the depth blocking of a GEMM); `matrix = false` sums every element
// over all observations in one sequential run instead (the nested-loop
// variant, glm_gradient_xyyhat.cuh:799-812 -- which in the reference forgets
// the elastic-net term; here both variants add it when `reg` is set).
template <typename T>
Tensor3D<T> gradient(const Tensor3D<T>& X, const Tensor3D<T>& M, const Tensor3D<T>& Y, double lambda,
                     double alpha, bool reg, bool matrix = true) {
    using A = arith_t<T>;
    const long nf = X.cols(), ntasks = X.rows(), nobs = X.sheets(), nt = M.rows();
    const long K = nf * nt;
    Tensor3D<T> grad(nf, nt, ntasks);
    const long panel = matrix ? 256 : std::max(1L, nobs);
    const long npanels = nobs > 0 ? (nobs + panel - 1) / panel : 0;
    for (long task = 0; task < ntasks; ++task) {
        std::vector<A> psum(static_cast<size_t>(std::max(1L, npanels)) * K, A(0));
#pragma omp parallel for schedule(dynamic, 1)
        for (long p = 0; p < npanels; ++p) {
            A* acc = psum.data() + p * K;
            std::vector<A> e(nt);
            const long o1 = std::min(nobs, (p + 1) * panel);
            for (long obs = p * panel; obs < o1; ++obs) {
                const T* x = &X(0, task, obs);
                for (long t = 0; t < nt; ++t) {
                    const T* m = &M(0, t, task);
                    A d = 0;
                    for (long f = 0; f < nf; ++f) d += up(m[f]) * up(x[f]);
                    e[t] = d - up(Y(t, task, obs));
                }
                for (long t = 0; t < nt; ++t)
                    for (long f = 0; f < nf; ++f) acc[t * nf + f] += e[t] * up(x[f]);
            }
        }
        const T lam_t = from_double<T>(lambda), alp_t = from_double<T>(alpha);
        const A lam = up(lam_t), alp = up(alp_t);
        const A two_lambda_one_minus_alpha = (A(2) * lam) * (A(1) - alp);
        const A lambda_alpha = lam * alp;
        for (long k = 0; k < K; ++k) {
            A s = 0;
            for (long p = 0; p < npanels; ++p) s += psum[p * K + k];
            A g = A(2) * s;
            const long t = k / nf, f = k % nf;
            if (reg && is_positive(lam_t)) {
                const T mv = M(f, t, task);
                if (is_positive(alp_t)) g += lambda_alpha * static_cast<A>(sign_of(mv));
                if (up(alp_t) < A(1)) g += two_lambda_one_minus_alpha * up(mv);
            }
            grad(f, t, task) = down<T>(g);
        }
    }
    return grad;
}

// loss = sum (Yhat - Y)^2 + lambda*(alpha*sum|M| + (1-alpha)*sum M^2), one
// element (glm_loss_myyhat.cuh:365-401 in gpu_algos), sums carried in arith_t.
template <typename T>
Tensor3D<T> loss(const Tensor3D<T>& M, const Tensor3D<T>& Y, const Tensor3D<T>& Yhat, double lambda, double alpha) {
    using A = arith_t<T>;
    Tensor3D<T> out(1, 1, 1);
    const long size_Y = Y.cols() * Y.rows() * Y.sheets(), size_M = M.cols() * M.rows() * M.sheets();
    const T* y = Y.data();
    const T* yh = Yhat.data();
    const T* m = M.data();
    A err = 0, l1 = 0, l2 = 0;
    for (long i = 0; i < size_Y; ++i) {
        const A e = up(yh[i]) - up(y[i]);
        err += e * e;
    }
    for (long i = 0; i < size_M; ++i) {
        const A v = up(m[i]);
        if constexpr (std::is_floating_point_v<A>) l1 += v < A(0) ? -v : v;
        else l1 += is_negative(m[i]) ? A(0) - v : v;
        l2 += v * v;
    }
    const A lam = up(from_double<T>(lambda)), alp = up(from_double<T>(alpha));
    out(0, 0, 0) = down<T>(err + lam * (alp * l1 + (A(1) - alp) * l2));
    return out;
}

// ---- typed bridge to the C ABI --------------------------------------------
#define GLMB_HOST_BRIDGE(T, CT, SFX)                                                                \
    inline int abi_predict(const T* X, const T* M, T* Yhat, long nf, long nt, long ntasks, long nobs, \
                           cudaStream_t s) {                                                        \
        return glmb_predict_##SFX(reinterpret_cast<const CT*>(X), reinterpret_cast<const CT*>(M),   \
                                  reinterpret_cast<CT*>(Yhat), nf, nt, ntasks, nobs,                \
                                  reinterpret_cast<glmb_stream_t>(s));                              \
    }                                                                                               \
    inline int abi_gradient(const T* X, const T* M, const T* Y, T* grad, T* Yhat, long nf, long nt, \
                            long ntasks, long nobs, double lambda, double alpha, uint32_t flags,    \
                            cudaStream_t s) {                                                       \
        return glmb_gradient_##SFX(reinterpret_cast<const CT*>(X), reinterpret_cast<const CT*>(M),  \
                                   reinterpret_cast<const CT*>(Y), reinterpret_cast<CT*>(grad),     \
                                   reinterpret_cast<CT*>(Yhat), nf, nt, ntasks, nobs, lambda, alpha, \
                                   flags, nullptr, 0, reinterpret_cast<glmb_stream_t>(s));          \
    }                                                                                               \
    inline int abi_loss(const T* M, const T* Y, const T* Yhat, T* loss, long nf, long nt, long ntasks,   \
                        long nobs, double lambda, double alpha, cudaStream_t s) {                   \
        return glmb_loss_##SFX(reinterpret_cast<const CT*>(M), reinterpret_cast<const CT*>(Y),      \
                               reinterpret_cast<const CT*>(Yhat), reinterpret_cast<CT*>(loss), nf,  \
                               nt, ntasks, nobs, lambda, alpha, nullptr, 0,                         \
                               reinterpret_cast<glmb_stream_t>(s));                                 \
    }                                                                                               \
    inline const char* abi_suffix(const T*) { return #SFX; }

GLMB_HOST_BRIDGE(__half, uint16_t, f16)
GLMB_HOST_BRIDGE(float, float, f32)
GLMB_HOST_BRIDGE(double, double, f64)
GLMB_HOST_BRIDGE(int8_t, int8_t, i8)
GLMB_HOST_BRIDGE(int16_t, int16_t, i16)
GLMB_HOST_BRIDGE(int32_t, int32_t, i32)
GLMB_HOST_BRIDGE(int64_t, int64_t, i64)
GLMB_HOST_BRIDGE(uint8_t, uint8_t, u8)
GLMB_HOST_BRIDGE(uint16_t, uint16_t, u16)
GLMB_HOST_BRIDGE(uint32_t, uint32_t, u32)
GLMB_HOST_BRIDGE(uint64_t, uint64_t, u64)
#undef GLMB_HOST_BRIDGE

}  // namespace glm_host
