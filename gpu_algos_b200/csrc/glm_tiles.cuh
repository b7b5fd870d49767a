// glm_tiles.cuh -- tiled float64 gradient for up to 16 targets (glm_tiles.cu).
#pragma once

#include "glm_common.cuh"

namespace glmb {

struct TilesPlan {
    int32_t ctas_per_task = 0;
    int64_t obs_per_cta = 0;
    size_t part_doubles = 0;
    size_t smem_bytes = 0;
};

// Shapes the tiled kernel serves: 0 < nfeatures <= 256 (even), 0 < ntargets <= 16,
// X 16-byte aligned.
bool tiles_f64_supported(int64_t nf, int64_t nt, int64_t ntasks, const void* X);
TilesPlan tiles_f64_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs);
// part: [task][nt*nf][ctas_per_task] doubles; status: one int, zero on entry.
int tiles_f64_launch(const TilesPlan& p, const double* X, const double* M, const double* Y, double* Yhat,
                     double* part, int* status, int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,
                     cudaStream_t stream);
// Overwrites the n outputs with NaN when *status is set (a bounded wait gave up).
int tiles_poison(const int* status, double* partial_out, double* grad, int64_t n, cudaStream_t stream);

}  // namespace glmb
