// glm_fit.cuh -- elastic-net proximal-gradient kernels (see glm_fit.cu).
#pragma once

#include "glm_common.cuh"

namespace glmb {

// Safety factor applied to the power-iteration estimate of the Lipschitz
// constant: power iteration approaches lambda_max from below.
constexpr double kPowerSafety = 1.05;

template <typename T>
int prox_step(T* beta, const T* g, int64_t n, double inv_L, double l1, cudaStream_t s);

template <typename T>
int prox_update(const double* P, T* beta, const double* lipschitz, int64_t K, int64_t ntasks,
                double lambda1, double lambda2, cudaStream_t s);

template <typename T>
int power_step(const double* P, T* v, double* norm, double* lipschitz, int64_t nf, int64_t ntasks,
               double lambda2, cudaStream_t s);

template <typename T>
int power_init(T* v, int64_t nf, int64_t ntasks, uint64_t seed, cudaStream_t s);

}  // namespace glmb
