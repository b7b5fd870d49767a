// glm_loss.cuh -- the GLM objective for every element type (glm_loss.cu).
#pragma once

#include "glm_common.cuh"

namespace glmb {

// Bytes of scratch loss_launch needs (the per-CTA partial sums).
size_t loss_workspace_bytes();

// loss[0] = sum_i (Yhat_i - Y_i)^2 + lambda (alpha sum |M| + (1 - alpha) sum M^2)
// over the nobs * ntasks * nt elements of Y / Yhat (Y == NULL: zeros) and the
// nf * nt * ntasks elements of M, with lambda and alpha taken in T (the
// reference's Number conversion).  float/double/half sum in double; integer
// types modulo 2^bits.  Deterministic (fixed reduction order).
template <typename T>
int loss_launch(const T* M, const T* Y, const T* Yhat, T* loss, int64_t nf, int64_t nt, int64_t ntasks,
                int64_t nobs, double lambda, double alpha, void* ws, size_t ws_bytes, cudaStream_t stream);

// The same scalar from a finished data term: `part` holds `nparts` partial
// sums of (Yhat - Y)^2 in double (the rows kernel's kRowsGradYhatLoss CTA
// partials), summed here in order before the model terms are added.
// float and double.
template <typename T>
int loss_from_partials_launch(const double* part, int64_t nparts, const T* M, int64_t size_M, T* loss,
                              double lambda, double alpha, cudaStream_t stream);

}  // namespace glmb
