// glm_rows.cuh -- fused row-streaming GLM kernel for float / double.
//
// One pass over X computes, for every row x = X[obs, task, :],
//     yhat_t = sum_f M[task, t, f] * x_f          (t < ntargets)
//     r_t    = yhat_t - Y[obs, task, t]
//     acc[t, f] += r_t * x_f
// so each byte of X is read from HBM once and yhat / r never leave the SM
// (yhat is stored only when asked for).  This replaces the reference's two
// launches, glm_predict_fixed_grid followed by glm_gradient_XYYhat_<algo>
// (include/cuda/kernels/glm/glm_gradient_xyyhat.cuh:659-782), which round-trip
// Yhat through HBM and re-read X with a stride of nfeatures*ntasks.
//
// Work layout.  A row of X (nf contiguous elements) is spread over a
// segment of S lanes (S a power of two <= 32); each lane owns CPL vectors of
// VEC elements, feature f = (c*S + lane_in_segment)*VEC + v, so a warp load
// instruction reads 32*VEC*sizeof(T) contiguous bytes (512 B for float4).
// A warp handles 32/S rows per step and U steps per loop iteration, issuing
// all U*CPL vector loads before the arithmetic that consumes them.  The dot
// product is finished with an xor-butterfly inside the segment, which leaves
// yhat in every lane of the segment.  Partial sums are carried in registers
// in the input precision for kFlushSteps iterations, then folded across the
// row groups of the warp and added into a per-warp double accumulator in
// shared memory.  At the end the warps of a CTA are summed in a fixed order
// and the CTA writes one double partial per (task, t, f); a second kernel
// (glm_finalize.cuh) sums the CTA partials in a fixed order.  Results are
// therefore deterministic for a given device and launch plan.
#pragma once

#include "glm_common.cuh"

namespace glmb {

enum RowsMode : int { kRowsGrad = 0, kRowsGradYhat = 1, kRowsPredict = 2 };

constexpr int kRowsWarps = 8;
constexpr int kRowsThreads = kRowsWarps * kWarp;
constexpr int kFlushIters = 8;

struct RowsArgs {
    const void* X;
    const void* M;
    const void* Y;  // may be NULL: all zeros
    void* Yhat;
    double* part;  // [task][nt*nf][ctas_per_task]
    int64_t nf;
    int64_t nt;
    int64_t ntasks;
    int64_t nobs;
    int64_t obs_per_cta;
    int32_t ctas_per_task;
    int32_t seg_log2;
};

template <typename T, int VEC, int CPL, int NT>
struct RowsShape {
    static constexpr int FPL = CPL * VEC;  // features per lane
    static constexpr int WORDS = FPL * int(sizeof(T)) / 4 + NT;
    static constexpr int U = (20 / WORDS) < 1 ? 1 : ((20 / WORDS) > 8 ? 8 : (20 / WORDS));
    static constexpr int SLOTS = NT * CPL * kWarp * VEC;  // doubles per warp in smem
    static constexpr size_t SMEM = size_t(kRowsWarps) * SLOTS * sizeof(double);
};

template <typename T, int VEC, int CPL, int NT, int MODE>
__global__ void __launch_bounds__(kRowsThreads) glm_rows_kernel(const RowsArgs a) {
    using D = typename Arith<T>::Dot;
    using Shape = RowsShape<T, VEC, CPL, NT>;
    constexpr int U = Shape::U;
    constexpr bool GRAD = MODE != kRowsPredict;
    extern __shared__ double smem_acc[];

    const T* __restrict__ X = static_cast<const T*>(a.X);
    const T* __restrict__ M = static_cast<const T*>(a.M);
    const T* __restrict__ Y = static_cast<const T*>(a.Y);
    T* __restrict__ Yhat = static_cast<T*>(a.Yhat);

    const int lane = threadIdx.x & (kWarp - 1);
    const int warp = threadIdx.x >> 5;
    const int S = 1 << a.seg_log2;
    const int R = kWarp >> a.seg_log2;  // rows per step
    const int grp = lane >> a.seg_log2;
    const int ls = lane & (S - 1);
    const int64_t task = blockIdx.x / a.ctas_per_task;
    const int64_t cta = blockIdx.x - task * a.ctas_per_task;
    const int64_t obs_begin = cta * a.obs_per_cta;
    const int64_t obs_end = min(a.nobs, obs_begin + a.obs_per_cta);
    const int nt = static_cast<int>(a.nt);
    const int64_t nf = a.nf;
    const int64_t ntasks = a.ntasks;

    // Model coefficients of this task, in registers.
    D m[NT][CPL][VEC];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int c = 0; c < CPL; ++c)
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
                const int64_t f = int64_t(c * S + ls) * VEC + v;
                m[t][c][v] = (t < nt && f < nf) ? to_arith<D>(M[(task * nt + t) * nf + f]) : D(0);
            }

    D acc[NT][CPL][VEC];
    double* wsm = smem_acc + size_t(warp) * Shape::SLOTS;
    if constexpr (GRAD) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int c = 0; c < CPL; ++c)
#pragma unroll
                for (int v = 0; v < VEC; ++v) acc[t][c][v] = D(0);
        for (int i = lane; i < Shape::SLOTS; i += kWarp) wsm[i] = 0.0;
    }

    // Fold the register partials of all row groups into the warp's double
    // accumulator (lanes of row group 0 own the shared-memory slots).
    auto flush = [&]() {
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int c = 0; c < CPL; ++c)
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    D val = acc[t][c][v];
                    for (int off = S; off < kWarp; off <<= 1)
                        val += __shfl_xor_sync(0xffffffffu, val, off);
                    if (grp == 0) wsm[((t * CPL + c) * kWarp + ls) * VEC + v] += double(val);
                    acc[t][c][v] = D(0);
                }
    };

    const int64_t warp_stride = int64_t(kRowsWarps) * U * R;
    int iters = 0;
    for (int64_t base = obs_begin + int64_t(warp) * U * R; base < obs_end; base += warp_stride) {
        T xv[U][CPL][VEC];
        D yv[U][NT];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t obs = base + int64_t(u) * R + grp;
            const bool ok = obs < obs_end;
            const int64_t row = obs * ntasks + task;
            const T* xrow = X + row * nf;
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const int64_t f0 = int64_t(c * S + ls) * VEC;
                if (ok && f0 < nf) {
                    VecLoad<T, VEC>::load(xrow + f0, xv[u][c]);
                } else {
#pragma unroll
                    for (int v = 0; v < VEC; ++v) xv[u][c][v] = T(0);
                }
            }
            if constexpr (GRAD) {
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    yv[u][t] = (ok && t < nt && Y != nullptr) ? to_arith<D>(Y[row * nt + t]) : D(0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t obs = base + int64_t(u) * R + grp;
            D r[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                D d = D(0);
#pragma unroll
                for (int c = 0; c < CPL; ++c)
#pragma unroll
                    for (int v = 0; v < VEC; ++v) d = fma(m[t][c][v], D(xv[u][c][v]), d);
                for (int off = S >> 1; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
                if constexpr (MODE != kRowsGrad) {
                    if (ls == 0 && t < nt && obs < obs_end) Yhat[(obs * ntasks + task) * nt + t] = T(d);
                }
                if constexpr (GRAD) r[t] = d - yv[u][t];
            }
            if constexpr (GRAD) {
#pragma unroll
                for (int t = 0; t < NT; ++t)
#pragma unroll
                    for (int c = 0; c < CPL; ++c)
#pragma unroll
                        for (int v = 0; v < VEC; ++v)
                            acc[t][c][v] = fma(r[t], D(xv[u][c][v]), acc[t][c][v]);
            }
        }
        if constexpr (GRAD) {
            if (++iters == kFlushIters) {
                flush();
                iters = 0;
            }
        }
    }
    if constexpr (GRAD) {
        flush();
        __syncthreads();
        // Sum the warps in a fixed order; one double per (t, f) for this CTA.
        const int64_t K = int64_t(nt) * nf;
        const int live = NT * CPL * S * VEC;
        for (int i = threadIdx.x; i < live; i += kRowsThreads) {
            const int v = i % VEC;
            const int l = (i / VEC) % S;
            const int c = (i / (VEC * S)) % CPL;
            const int t = i / (VEC * S * CPL);
            const int64_t f = int64_t(c * S + l) * VEC + v;
            if (t >= nt || f >= nf) continue;
            const int slot = ((t * CPL + c) * kWarp + l) * VEC + v;
            double s = 0.0;
#pragma unroll
            for (int w = 0; w < kRowsWarps; ++w) s += smem_acc[size_t(w) * Shape::SLOTS + slot];
            a.part[(task * K + int64_t(t) * nf + f) * a.ctas_per_task + cta] = s;
        }
    }
}

// Plan of one rows launch.
struct RowsPlan {
    bool ok = false;        // shape is served by the rows kernel
    int vec = 1, cpl = 1, ntmax = 1, seg_log2 = 5;
    int32_t ctas_per_task = 0;
    int64_t obs_per_cta = 0;
    size_t part_doubles = 0;
};

// Choose VEC / CPL / NT / S for (T, nf, nt) and the grid; see glm_rows.cu.
template <typename T>
RowsPlan rows_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, bool vec_aligned,
                   bool grad);

template <typename T>
int rows_launch(const RowsPlan& p, int mode, const RowsArgs& args, cudaStream_t stream);

}  // namespace glmb
