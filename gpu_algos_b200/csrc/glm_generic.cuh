// glm_generic.cuh -- kernels for every element type and shape, and the
// deterministic cross-CTA reduction shared by all gradient paths.
#pragma once

#include "glm_common.cuh"

namespace glmb {

// Bytes of scratch the generic gradient path needs.
template <typename T>
size_t generic_workspace_bytes(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs);

// Yhat = X.M for any element type (one thread per output element).
template <typename T>
int generic_predict(const T* X, const T* M, T* Yhat, int64_t nf, int64_t nt, int64_t ntasks,
                    int64_t nobs, cudaStream_t stream);

// Two-pass gradient for any element type and shape: residuals E = Yhat - Y
// into scratch, then per-(task, feature-block, obs-split) sums of E*X, then
// the fixed-order reduction over splits.  With partial_out != NULL the
// reduction writes sum (Yhat - Y) X as double instead of the gradient.
// With `fin` set, fin(fin_ctx, part, nparts) replaces that reduction: part is
// laid out [e][nparts] in the Acc type (double for float/double inputs).
// `logistic` (floating types): residuals sigmoid(x.m) - y, predictions
// sigmoid(x.m), the gradient of the logistic negative log-likelihood.
using PartsFinisher = int (*)(void* ctx, const void* part, int64_t nparts);
template <typename T>
int generic_gradient(const T* X, const T* M, const T* Y, T* grad, T* Yhat, double* partial_out,
                     int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, double lambda,
                     double alpha, bool reg, void* ws, size_t ws_bytes, cudaStream_t stream,
                     PartsFinisher fin = nullptr, void* fin_ctx = nullptr, bool logistic = false);

// Reduction of per-part sums part[e * nparts + c] over c in a fixed order, one
// warp per output element e < total, then either
//   grad[e] = 2*sum + elastic-net term   (partial_out == NULL), or
//   partial_out[e] = sum                 (double).
template <typename T, typename P>
int finalize_launch(const P* part, int64_t nparts, int64_t total, const T* M, T* grad,
                    double* partial_out, double lambda, double alpha, bool reg,
                    cudaStream_t stream);

}  // namespace glmb
