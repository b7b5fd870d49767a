// glm_dense.cuh -- float32 dense-shape gradient on tcgen05 tensor cores (glm_dense.cu).
#pragma once

#include "glm_common.cuh"

namespace glmb {

struct DensePlan {
    int64_t nt_pad = 0, obs_per_split = 0, nsplit = 0;
    size_t r_bytes = 0, p_bytes = 0, mlo_bytes = 0, ws_bytes = 0;
};

// X and M 16-byte aligned, nfeatures a multiple of 4 (TMA row strides), >= 32.
bool dense_f32_supported(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, const void* X, const void* M);
DensePlan dense_f32_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs);
// ws: at least plan.ws_bytes, 256-byte aligned.
int dense_f32_gradient(const DensePlan& p, const float* X, const float* M, const float* Y, float* grad,
                       float* Yhat, double* partial_out, int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,
                       double lambda, double alpha, bool reg, void* ws, cudaStream_t stream);

}  // namespace glmb
