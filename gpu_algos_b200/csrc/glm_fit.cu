// glm_fit.cu -- elastic-net proximal-gradient (ISTA) kernels.
//
// The reference ships the elastic-net gradient term but no optimizer; these
// kernels implement the proximal step from the mathematics (Daubechies,
// Defrise & De Mol 2004; Beck & Teboulle 2009) in the reference's loss
// convention  sum (yhat - y)^2 + lambda1*|M|_1 + lambda2*|M|^2.
// Every kernel is elementwise over (task, target, feature) or one block per
// task, reads its step size from device memory and never synchronises the
// host, so a whole fit is one stream of launches (and can be captured).
#include <cmath>

#include "glm_common.cuh"
#include "glm_fit.cuh"

namespace glmb {

namespace {

__device__ __forceinline__ double soft_threshold(double z, double t) {
    const double a = fabs(z) - t;
    if (a <= 0.0) return 0.0;
    return z > 0.0 ? a : -a;
}

// SplitMix64 (Steele, Lea & Flood 2014): the i-th output of the generator
// seeded with `seed`, mapped from its top 53 bits to [-1, 1).
__device__ __forceinline__ double splitmix_uniform(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return 2.0 * (double(z >> 11) * (1.0 / 9007199254740992.0)) - 1.0;
}

constexpr int kFitThreads = 256;

// Fixed-order block sum of one double per thread (result valid in thread 0).
__device__ double block_sum(double v, double* red) {
#pragma unroll
    for (int off = kWarp / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int lane = threadIdx.x & (kWarp - 1), warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < int(blockDim.x >> 5); ++w) s += red[w];
    __syncthreads();
    return s;
}

template <typename T>
__global__ void __launch_bounds__(kFitThreads)
    prox_step_kernel(T* __restrict__ beta, const T* __restrict__ g, int64_t n, double inv_L, double l1) {
    const double thr = l1 * inv_L;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const double z = double(beta[i]) - double(g[i]) * inv_L;
        beta[i] = T(soft_threshold(z, thr));
    }
}

// g = 2P + 2*lambda2*beta in T arithmetic (the regularised gradient with
// alpha = 0), then beta <- S(beta - g/L[task], lambda1/L[task]).
template <typename T>
__global__ void __launch_bounds__(kFitThreads)
    prox_update_kernel(const double* __restrict__ P, T* __restrict__ beta,
                       const double* __restrict__ lipschitz, int64_t K, int64_t total, double lambda1,
                       double lambda2) {
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += stride) {
        const double inv_L = 1.0 / lipschitz[e / K];
        const T b = beta[e];
        const T g = finalize_value<T>(P[e], b, lambda2, 0.0, true);
        const double z = double(b) - double(g) * inv_L;
        beta[e] = T(soft_threshold(z, lambda1 * inv_L));
    }
}

// One block per task: g = 2P (T arithmetic), norm = |g|, v = g / norm,
// lipschitz = safety*norm + 2*lambda2.
template <typename T>
__global__ void __launch_bounds__(kFitThreads)
    power_step_kernel(const double* __restrict__ P, T* __restrict__ v, double* __restrict__ norm,
                      double* __restrict__ lipschitz, int64_t nf, double lambda2, double safety) {
    __shared__ double red[kFitThreads / kWarp];
    __shared__ double inv_s;
    const int64_t task = blockIdx.x;
    const double* p = P + task * nf;
    double s = 0.0;
    for (int64_t f = threadIdx.x; f < nf; f += blockDim.x) {
        const double g = double(finalize_value<T>(p[f], T(0), 0.0, 0.0, false));
        s += g * g;
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) {
        const double nrm = sqrt(s);
        norm[task] = nrm;
        lipschitz[task] = safety * nrm + 2.0 * lambda2;
        inv_s = nrm > 0.0 ? 1.0 / nrm : 0.0;
    }
    __syncthreads();
    const double inv = inv_s;
    for (int64_t f = threadIdx.x; f < nf; f += blockDim.x) {
        const double g = double(finalize_value<T>(p[f], T(0), 0.0, 0.0, false));
        v[task * nf + f] = T(g * inv);
    }
}

// One block per task: v0 = SplitMix64 uniforms rounded to T, normalised.
template <typename T>
__global__ void __launch_bounds__(kFitThreads)
    power_init_kernel(T* __restrict__ v, int64_t nf, uint64_t seed) {
    __shared__ double red[kFitThreads / kWarp];
    __shared__ double inv_s;
    const int64_t task = blockIdx.x;
    double s = 0.0;
    for (int64_t f = threadIdx.x; f < nf; f += blockDim.x) {
        const double x = double(T(splitmix_uniform(seed, uint64_t(task * nf + f))));
        s += x * x;
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) inv_s = s > 0.0 ? 1.0 / sqrt(s) : 0.0;
    __syncthreads();
    const double inv = inv_s;
    for (int64_t f = threadIdx.x; f < nf; f += blockDim.x) {
        const double x = double(T(splitmix_uniform(seed, uint64_t(task * nf + f))));
        v[task * nf + f] = T(x * inv);
    }
}

inline unsigned elem_grid(int64_t n) {
    const int64_t cap = int64_t(sm_count()) * 8;
    return unsigned(std::max<int64_t>(1, std::min<int64_t>(cap, (n + kFitThreads - 1) / kFitThreads)));
}

}  // namespace

template <typename T>
int prox_step(T* beta, const T* g, int64_t n, double inv_L, double l1, cudaStream_t s) {
    if (n == 0) return GLMB_OK;
    prox_step_kernel<T><<<elem_grid(n), kFitThreads, 0, s>>>(beta, g, n, inv_L, l1);
    count_launch();
    return launch_status();
}

template <typename T>
int prox_update(const double* P, T* beta, const double* lipschitz, int64_t K, int64_t ntasks,
                double lambda1, double lambda2, cudaStream_t s) {
    const int64_t total = K * ntasks;
    if (total == 0) return GLMB_OK;
    prox_update_kernel<T><<<elem_grid(total), kFitThreads, 0, s>>>(P, beta, lipschitz, K, total,
                                                                    lambda1, lambda2);
    count_launch();
    return launch_status();
}

template <typename T>
int power_step(const double* P, T* v, double* norm, double* lipschitz, int64_t nf, int64_t ntasks,
               double lambda2, cudaStream_t s) {
    if (ntasks == 0) return GLMB_OK;
    power_step_kernel<T><<<unsigned(ntasks), kFitThreads, 0, s>>>(P, v, norm, lipschitz, nf, lambda2,
                                                                   kPowerSafety);
    count_launch();
    return launch_status();
}

template <typename T>
int power_init(T* v, int64_t nf, int64_t ntasks, uint64_t seed, cudaStream_t s) {
    if (ntasks == 0 || nf == 0) return GLMB_OK;
    power_init_kernel<T><<<unsigned(ntasks), kFitThreads, 0, s>>>(v, nf, seed);
    count_launch();
    return launch_status();
}

#define GLMB_INSTANTIATE_FIT(T)                                                                    \
    template int prox_step<T>(T*, const T*, int64_t, double, double, cudaStream_t);                \
    template int prox_update<T>(const double*, T*, const double*, int64_t, int64_t, double, double, \
                                cudaStream_t);                                                     \
    template int power_step<T>(const double*, T*, double*, double*, int64_t, int64_t, double,      \
                               cudaStream_t);                                                      \
    template int power_init<T>(T*, int64_t, int64_t, uint64_t, cudaStream_t);

GLMB_INSTANTIATE_FIT(float)
GLMB_INSTANTIATE_FIT(double)

}  // namespace glmb
