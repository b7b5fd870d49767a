// glm_loss.cu -- the GLM objective, the counterpart of the reference's
// Glm_loss_myyhat kernel class (include/cuda/kernels/glm/glm_loss_myyhat.cuh:
// GPU kernel :100-158, host definition :365-401):
//
//   loss = sum_i (Yhat_i - Y_i)^2 + lambda (alpha sum |M| + (1 - alpha) sum M^2)
//
// over all targets, tasks and observations.  Two launches: a streaming pass
// over Y and Yhat (HBM-bound: 2 sizeof(T) bytes per element, grid = SMs x 4
// CTAs, each CTA's sum to scratch), then one CTA sums the CTA partials in a
// fixed order, adds the model terms (one pass over M) and writes the scalar.
// When the gradient's rows kernel has already summed the squared residuals
// (glmb_gradient_loss_*), only the second launch runs, on its partials.
// float/double/half carry the sums in double (the reference sums in its
// Number type; double is closer to the exact sum); integer types compute
// modulo 2^bits in their unsigned arithmetic type, which is what the
// reference's Number arithmetic gives (bit-exact).
#include <algorithm>

#include "glm_loss.cuh"

namespace glmb {

namespace {

constexpr int kLossThreads = 256;
constexpr int kLossMaxCtas = 1024;
constexpr int kFinalThreads = 1024;

// Type the sums are carried in.
template <typename T>
struct LossAcc {
    using type = typename Arith<T>::Acc;  // integers: modular unsigned
};
template <>
struct LossAcc<float> {
    using type = double;
};
template <>
struct LossAcc<__half> {
    using type = double;
};
template <>
struct LossAcc<__nv_bfloat16> {
    using type = double;
};

template <typename L, typename T>
__device__ __forceinline__ L load_as(const T* p, int64_t i) {
    return p == nullptr ? L(0) : to_arith<L>(p[i]);
}

// |m| in the sum type: integers negate modulo 2^bits, as the reference's abs
// of a Number followed by Number arithmetic does.
template <typename L, typename T>
__device__ __forceinline__ L abs_as(T m) {
    if constexpr (std::is_floating_point_v<L>) {
        const L v = to_arith<L>(m);
        return v < L(0) ? -v : v;
    } else if constexpr (std::is_unsigned_v<T>) {
        return L(m);
    } else {
        return m < T(0) ? L(0) - L(m) : L(m);
    }
}

template <typename L>
__device__ __forceinline__ L warp_sum(L v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Per-CTA sums of (Yhat - Y)^2; warps and threads combined in a fixed order.
template <typename T, typename L>
__global__ void __launch_bounds__(kLossThreads)
    glm_loss_partial_kernel(const T* __restrict__ Y, const T* __restrict__ Yhat, L* __restrict__ part, int64_t n) {
    __shared__ L red[kLossThreads / 32];
    L s = L(0);
    const int64_t stride = int64_t(gridDim.x) * kLossThreads;
#pragma unroll 4
    for (int64_t i = int64_t(blockIdx.x) * kLossThreads + threadIdx.x; i < n; i += stride) {
        const L e = load_as<L>(Yhat, i) - load_as<L>(Y, i);
        s += e * e;
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        L t = L(0);
#pragma unroll
        for (int w = 0; w < kLossThreads / 32; ++w) t += red[w];
        part[blockIdx.x] = t;
    }
}

// One CTA: the partials in order, the model terms, the scalar.
template <typename T, typename L>
__global__ void __launch_bounds__(kFinalThreads)
    glm_loss_final_kernel(const L* __restrict__ part, int nparts, const T* __restrict__ M, int64_t size_M,
                          T* __restrict__ loss, double lambda, double alpha) {
    __shared__ L red[3][kFinalThreads / 32];
    L err = L(0), l1 = L(0), l2 = L(0);
    for (int i = threadIdx.x; i < nparts; i += kFinalThreads) err += part[i];
    for (int64_t i = threadIdx.x; i < size_M; i += kFinalThreads) {
        const T m = M[i];
        const L v = to_arith<L>(m);
        l1 += abs_as<L>(m);
        l2 += v * v;
    }
    err = warp_sum(err);
    l1 = warp_sum(l1);
    l2 = warp_sum(l2);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        red[0][w] = err;
        red[1][w] = l1;
        red[2][w] = l2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        L e = L(0), a1 = L(0), a2 = L(0);
        for (int k = 0; k < kFinalThreads / 32; ++k) {
            e += red[0][k];
            a1 += red[1][k];
            a2 += red[2][k];
        }
        // lambda and alpha in the Number type (glm_loss_myyhat.cuh:317-324), then
        // lambda * (alpha * l1 + (1 - alpha) * l2) (:395)
        const L lam = to_arith<L>(from_double<T>(lambda)), alp = to_arith<L>(from_double<T>(alpha));
        const L reg = lam * (alp * a1 + (L(1) - alp) * a2);
        loss[0] = from_arith<T>(e + reg);
    }
}

}  // namespace

size_t loss_workspace_bytes() { return round_up(size_t(kLossMaxCtas) * sizeof(double), 256); }

template <typename T>
int loss_launch(const T* M, const T* Y, const T* Yhat, T* loss, int64_t nf, int64_t nt, int64_t ntasks,
                int64_t nobs, double lambda, double alpha, void* ws, size_t ws_bytes, cudaStream_t stream) {
    using L = typename LossAcc<T>::type;
    const int64_t n = nobs * ntasks * nt, size_M = nf * nt * ntasks;
    if (loss == nullptr || (n > 0 && Yhat == nullptr) || (size_M > 0 && M == nullptr)) return GLMB_ERR_INVALID_VALUE;
    Scratch sc(ws, ws_bytes, loss_workspace_bytes(), stream);
    if (sc.status() != GLMB_OK) return sc.status();
    L* part = sc.as<L>();
    int nparts = 0;
    if (n > 0) {
        nparts = int(std::min<int64_t>({int64_t(kLossMaxCtas), int64_t(sm_count()) * 4,
                                        (n + kLossThreads - 1) / kLossThreads}));
        glm_loss_partial_kernel<T, L><<<nparts, kLossThreads, 0, stream>>>(Y, Yhat, part, n);
        count_launch();
        const int st = launch_status();
        if (st != GLMB_OK) return st;
    }
    glm_loss_final_kernel<T, L><<<1, kFinalThreads, 0, stream>>>(part, nparts, M, size_M, loss, lambda, alpha);
    count_launch();
    return launch_status();
}

template <typename T>
int loss_from_partials_launch(const double* part, int64_t nparts, const T* M, int64_t size_M, T* loss,
                              double lambda, double alpha, cudaStream_t stream) {
    static_assert(std::is_same_v<typename LossAcc<T>::type, double>, "double data term");
    if (loss == nullptr || nparts < 0 || nparts > int64_t(0x7fffffff) || (nparts > 0 && part == nullptr) ||
        (size_M > 0 && M == nullptr))
        return GLMB_ERR_INVALID_VALUE;
    glm_loss_final_kernel<T, double><<<1, kFinalThreads, 0, stream>>>(part, int(nparts), M, size_M, loss, lambda,
                                                                     alpha);
    count_launch();
    return launch_status();
}
template int loss_from_partials_launch<float>(const double*, int64_t, const float*, int64_t, float*, double, double,
                                              cudaStream_t);
template int loss_from_partials_launch<double>(const double*, int64_t, const double*, int64_t, double*, double,
                                               double, cudaStream_t);

#define GLMB_INSTANTIATE_LOSS(T)                                                                        \
    template int loss_launch<T>(const T*, const T*, const T*, T*, int64_t, int64_t, int64_t, int64_t, double, \
                                double, void*, size_t, cudaStream_t);
GLMB_INSTANTIATE_LOSS(__half)
GLMB_INSTANTIATE_LOSS(__nv_bfloat16)
GLMB_INSTANTIATE_LOSS(float)
GLMB_INSTANTIATE_LOSS(double)
GLMB_INSTANTIATE_LOSS(int8_t)
GLMB_INSTANTIATE_LOSS(int16_t)
GLMB_INSTANTIATE_LOSS(int32_t)
GLMB_INSTANTIATE_LOSS(int64_t)
GLMB_INSTANTIATE_LOSS(uint8_t)
GLMB_INSTANTIATE_LOSS(uint16_t)
GLMB_INSTANTIATE_LOSS(uint32_t)
GLMB_INSTANTIATE_LOSS(uint64_t)
#undef GLMB_INSTANTIATE_LOSS

}  // namespace glmb
