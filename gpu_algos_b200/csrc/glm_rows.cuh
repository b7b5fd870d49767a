// glm_rows.cuh -- fused row-streaming GLM kernel for float / double / half /
// bfloat16 (16-bit types: float arithmetic on packed loads of 2-8 values,
// half the HBM bytes of float per feature).
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
// A warp handles 32/S rows per step and U steps per batch, issuing all
// U*CPL vector loads of the next batch before the arithmetic of the current
// one.  Partial sums are carried in registers in the input precision for
// kFlushIters batches, then folded across the row groups of the warp and
// added into a per-warp double accumulator in shared memory.  At the end the
// warps of a CTA are summed in a fixed order and the CTA writes one double
// partial per (task, t, f); glm_finalize_kernel (glm_generic.cu) sums the
// CTA partials in a fixed order.  Results are therefore deterministic for a
// given device and launch plan.
#pragma once

#include "glm_common.cuh"

namespace glmb {

// kRowsGradLogit*: logistic link -- the residual is sigmoid(x.m) - y, scaled
// by 1/2 so that the finalize's 2*sum gives the gradient of the logistic
// negative log-likelihood; the written prediction is sigmoid(x.m).
// kRowsGradYhatLoss: kRowsGradYhat that also sums the squared residuals of
// its rows (in double) into one partial per CTA, the objective's data term,
// so the loss costs no second pass over Y and Yhat.
enum RowsMode : int {
    kRowsGrad = 0,
    kRowsGradYhat = 1,
    kRowsPredict = 2,
    kRowsGradLogit = 3,
    kRowsGradLogitYhat = 4,
    kRowsGradYhatLoss = 5,
    kRowsModes = 6
};


constexpr int kRowsWarps = 8;
constexpr int kRowsThreads = kRowsWarps * kWarp;
constexpr int kFlushIters = 8;

struct RowsArgs {
    const void* X;
    const void* M;
    const void* Y;  // may be NULL: all zeros
    void* Yhat;
    double* part;  // [task][nt*nf][part_stride]
    int64_t nf;
    int64_t nt;
    int64_t ntasks;
    int64_t nobs;
    int64_t obs_per_cta;
    int64_t part_stride;  // partials per (task, t, f): >= ctas_per_task
    int64_t part_offset;  // column of this launch's first CTA
    int32_t ctas_per_task;
    int32_t seg_log2;
    double* loss_part;  // kRowsGradYhatLoss: sum of r^2 per CTA, [task][ctas_per_task]
};

template <typename T, int VEC, int CPL, int NT>
struct RowsShape {
    static constexpr int FPL = CPL * VEC;  // features per lane
    static constexpr int WORDS = FPL * int(sizeof(T)) / 4 + NT;
    // register words a batch may take; half rows carry half the bytes per
    // register, so twice as many of them keep as many bytes in flight; float
    // rows of 16 features per lane (512 across a warp) take two rows per
    // batch, so a warp keeps two 2 KB rows in flight rather than one
    static constexpr bool LONG_F32 = sizeof(T) == 4 && FPL == 16 && NT == 1;
    static constexpr int U_BUDGET = sizeof(T) == 2 ? 40 : (LONG_F32 ? 34 : 20);
    static constexpr int U_RAW = U_BUDGET / WORDS;
    // resident CTAs per SM the register allocation must leave room for (the
    // two-row batches of long float rows pay off only at two CTAs per SM)
    static constexpr int MIN_CTAS = LONG_F32 ? 2 : 1;
    // rows (or row steps) per batch: a power of two in [1, 8]
    static constexpr int U = U_RAW >= 8 ? 8 : (U_RAW >= 4 ? 4 : (U_RAW >= 2 ? 2 : 1));
    static constexpr int LOG2U = U == 8 ? 3 : (U == 4 ? 2 : (U == 2 ? 1 : 0));
    static constexpr int SLOTS = NT * CPL * kWarp * VEC;  // doubles per warp in smem
    static constexpr size_t SMEM = size_t(kRowsWarps) * SLOTS * sizeof(double);
};

// Register image of one lane's VEC consecutive elements of a row and of the
// matching model coefficients, with the two operations the kernel applies to
// them: the dot-product step d += m . x (elements in order) and the gradient
// step acc += r * x.  Generic types hold the elements themselves, in the
// arithmetic type D.
template <typename T, int VEC>
struct XRegs {
    static constexpr int N = VEC;
    using W = T;
    template <typename D>
    using MW = D;
    template <typename D>
    static constexpr int MN = VEC;
    __device__ __forceinline__ static void load(const T* p, W (&w)[N]) { VecLoad<T, VEC>::load(p, w); }
    template <typename D>
    __device__ __forceinline__ static void load_m(const T* mrow, int64_t f0, int64_t nf, bool ok, D (&m)[VEC]) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) m[v] = (ok && f0 + v < nf) ? to_arith<D>(mrow[f0 + v]) : D(0);
    }
    template <typename D>
    __device__ __forceinline__ static D dot(const D (&m)[VEC], const W (&w)[N], D d) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) d = fma(m[v], D(w[v]), d);
        return d;
    }
    // accumulators of the gradient step: one D per element
    template <typename D>
    using AW = D;
    template <typename D>
    static constexpr int AN = VEC;
    template <typename D>
    using RW = D;
    template <typename D>
    __device__ __forceinline__ static RW<D> prep(D r) {
        return r;
    }
    template <typename D>
    __device__ __forceinline__ static D acc_get(const D (&acc)[VEC], int v) {
        return acc[v];
    }
    template <typename D>
    __device__ __forceinline__ static void axpy(D r, const W (&w)[N], D (&acc)[VEC]) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] = fma(r, D(w[v]), acc[v]);
    }
};

// 16-bit float rows (__half, bfloat16), VEC >= 2: elements and coefficients
// stay packed in pairs in 32-bit words (element 2i in the low half of word
// i), so a batch of such rows takes half the registers of a batch of float
// rows.  The dot step is the mixed-precision fma.rn.f32.{f16,bf16}
// (16-bit x 16-bit + f32, rounded once): the product of two 16-bit floats is
// exact in float, so it equals converting both operands and a float FMA,
// with no conversion instruction.  The gradient step converts each pair and
// updates two float accumulators with one packed fma.rn.f32x2 (per element
// the same rounding as a scalar FMA).  A 16-bit row carries the float row's
// arithmetic on half the bytes, so these instruction counts (one per
// element for the dot, one and a half for the gradient, against two and two)
// decide whether it keeps up with HBM.
template <typename T>
__device__ __forceinline__ float fma_half16_pair(uint32_t m, uint32_t x, float d) {
    if constexpr (std::is_same_v<T, __half>) {
        asm("{\n\t.reg .f16 ml, mh, xl, xh;\n\t"
            "mov.b32 {ml, mh}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
            "fma.rn.f32.f16 %0, ml, xl, %0;\n\tfma.rn.f32.f16 %0, mh, xh, %0;\n\t}"
            : "+f"(d)
            : "r"(m), "r"(x));
    } else {
        asm("{\n\t.reg .b16 ml, mh, xl, xh;\n\t"
            "mov.b32 {ml, mh}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
            "fma.rn.f32.bf16 %0, ml, xl, %0;\n\tfma.rn.f32.bf16 %0, mh, xh, %0;\n\t}"
            : "+f"(d)
            : "r"(m), "r"(x));
    }
    return d;
}
// acc (two floats, element 2i in the low half) += rr (r in both halves) * x
template <typename T>
__device__ __forceinline__ void axpy_half16_pair(uint64_t rr, uint32_t x, uint64_t& acc) {
    if constexpr (std::is_same_v<T, __half>) {
        asm("{\n\t.reg .f16 xl, xh;\n\t.reg .f32 x0, x1;\n\t.reg .b64 xx;\n\t"
            "mov.b32 {xl, xh}, %2;\n\tcvt.f32.f16 x0, xl;\n\tcvt.f32.f16 x1, xh;\n\t"
            "mov.b64 xx, {x0, x1};\n\tfma.rn.f32x2 %0, %1, xx, %0;\n\t}"
            : "+l"(acc)
            : "l"(rr), "r"(x));
    } else {
        // bfloat16 -> float is exact: the 16 bits become the high half of the float
        asm("{\n\t.reg .b32 x0, x1;\n\t.reg .b64 xx;\n\t"
            "shl.b32 x0, %2, 16;\n\tand.b32 x1, %2, 0xffff0000;\n\t"
            "mov.b64 xx, {x0, x1};\n\tfma.rn.f32x2 %0, %1, xx, %0;\n\t}"
            : "+l"(acc)
            : "l"(rr), "r"(x));
    }
}
template <typename T, int VEC>
    requires kHalf16<T>
struct XRegs<T, VEC> {
    static_assert(VEC == 2 || VEC == 4 || VEC == 8, "packed 16-bit vectors");
    static constexpr int N = VEC / 2;
    using W = uint32_t;
    template <typename D>
    using MW = uint32_t;
    template <typename D>
    static constexpr int MN = N;
    __device__ __forceinline__ static void load(const T* p, W (&w)[N]) {
        if constexpr (N == 4) {
            asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                         : "l"(p));
        } else if constexpr (N == 2) {
            asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
        } else {
            asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
        }
    }
    template <typename D>
    __device__ __forceinline__ static void load_m(const T* mrow, int64_t f0, int64_t nf, bool ok, uint32_t (&m)[N]) {
        const unsigned short* bits = reinterpret_cast<const unsigned short*>(mrow);
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const unsigned short lo = (ok && f0 + 2 * i < nf) ? bits[f0 + 2 * i] : 0;
            const unsigned short hi = (ok && f0 + 2 * i + 1 < nf) ? bits[f0 + 2 * i + 1] : 0;
            m[i] = uint32_t(lo) | (uint32_t(hi) << 16);
        }
    }
    template <typename D>
    __device__ __forceinline__ static D dot(const uint32_t (&m)[N], const W (&w)[N], D d) {
#pragma unroll
        for (int i = 0; i < N; ++i) d = fma_half16_pair<T>(m[i], w[i], d);
        return d;
    }
    // accumulators: float pairs in 64-bit registers, the operands of
    // fma.rn.f32x2; the residual is packed into both halves once per row
    template <typename D>
    using AW = uint64_t;
    template <typename D>
    static constexpr int AN = N;
    template <typename D>
    using RW = uint64_t;
    template <typename D>
    __device__ __forceinline__ static uint64_t prep(D r) {
        const uint64_t b = __float_as_uint(r);
        return b | (b << 32);
    }
    template <typename D>
    __device__ __forceinline__ static D acc_get(const uint64_t (&acc)[N], int v) {
        const uint64_t p = acc[v >> 1];
        return __uint_as_float(static_cast<uint32_t>((v & 1) ? (p >> 32) : p));
    }
    template <typename D>
    __device__ __forceinline__ static void axpy(uint64_t rr, const W (&w)[N], uint64_t (&acc)[N]) {
#pragma unroll
        for (int i = 0; i < N; ++i) axpy_half16_pair<T>(rr, w[i], acc[i]);
    }
};
template <typename T>
    requires kHalf16<T>
struct XRegs<T, 1> {
    static constexpr int N = 1;
    using W = T;
    template <typename D>
    using MW = D;
    template <typename D>
    static constexpr int MN = 1;
    __device__ __forceinline__ static void load(const T* p, W (&w)[1]) { VecLoad<T, 1>::load(p, w); }
    template <typename D>
    __device__ __forceinline__ static void load_m(const T* mrow, int64_t f0, int64_t nf, bool ok, D (&m)[1]) {
        m[0] = (ok && f0 < nf) ? to_arith<D>(mrow[f0]) : D(0);
    }
    template <typename D>
    __device__ __forceinline__ static D dot(const D (&m)[1], const W (&w)[1], D d) {
        return fma(m[0], D(half16_to_float(w[0])), d);
    }
    template <typename D>
    using AW = D;
    template <typename D>
    static constexpr int AN = 1;
    template <typename D>
    using RW = D;
    template <typename D>
    __device__ __forceinline__ static RW<D> prep(D r) {
        return r;
    }
    template <typename D>
    __device__ __forceinline__ static D acc_get(const D (&acc)[1], int) {
        return acc[0];
    }
    template <typename D>
    __device__ __forceinline__ static void axpy(D r, const W (&w)[1], D (&acc)[1]) {
        acc[0] = fma(r, D(half16_to_float(w[0])), acc[0]);
    }
};

// FULL: one row per warp (S = 32).  The U rows of a batch are then reduced
// together: a transposed butterfly halves the set of rows a lane carries at
// each of the first log2(U) exchange steps, so a batch of U rows costs
// (U-1) + (5-log2 U) shuffles plus U broadcasts of the residual instead of
// 5U shuffles; afterwards lane L holds the complete dot product of row
// L >> (5 - log2 U).  Without FULL (S < 32, short rows) a warp carries 32/S
// rows per step and each segment finishes its own butterfly.
//
// Loads are double-buffered in registers: the loads of batch i+1 are issued
// before the arithmetic of batch i, so every warp keeps one batch of X in
// flight while it computes.
template <typename T, int VEC, int CPL, int NT, int MODE, bool FULL>
__global__ void __launch_bounds__(kRowsThreads, RowsShape<T, VEC, CPL, NT>::MIN_CTAS) glm_rows_kernel(const RowsArgs a) {
    using D = typename Arith<T>::Dot;
    using Shape = RowsShape<T, VEC, CPL, NT>;
    using XR = XRegs<T, VEC>;
    using XW = typename XR::W;
    constexpr int XN = XR::N;
    constexpr int U = Shape::U;
    constexpr int LOG2U = Shape::LOG2U;
    constexpr bool GRAD = MODE != kRowsPredict;
    constexpr bool LOGIT = MODE == kRowsGradLogit || MODE == kRowsGradLogitYhat;
    constexpr bool WRITE =
        MODE == kRowsGradYhat || MODE == kRowsPredict || MODE == kRowsGradLogitYhat || MODE == kRowsGradYhatLoss;
    constexpr bool LOSS = MODE == kRowsGradYhatLoss;
    extern __shared__ double smem_acc[];

    const T* __restrict__ X = static_cast<const T*>(a.X);
    const T* __restrict__ M = static_cast<const T*>(a.M);
    const T* __restrict__ Y = static_cast<const T*>(a.Y);
    T* __restrict__ Yhat = static_cast<T*>(a.Yhat);

    pdl_allow_dependents();  // the reduction of this launch's partials may start launching
    const int lane = threadIdx.x & (kWarp - 1);
    const int warp = threadIdx.x >> 5;
    const int seg_log2 = FULL ? 5 : a.seg_log2;
    const int S = 1 << seg_log2;
    const int R = kWarp >> seg_log2;  // rows per step
    const int grp = lane >> seg_log2;
    const int ls = lane & (S - 1);
    const int64_t task = blockIdx.x / a.ctas_per_task;
    const int64_t cta = blockIdx.x - task * a.ctas_per_task;
    const int64_t obs_begin = cta * a.obs_per_cta;
    const int64_t obs_end = min(a.nobs, obs_begin + a.obs_per_cta);
    const int nt = static_cast<int>(a.nt);
    const int64_t nf = a.nf;
    const int64_t ntasks = a.ntasks;
    // FULL: the batch row whose dot product this lane completes
    const int u_mine = FULL ? (lane >> (5 - LOG2U)) : 0;

    // Model coefficients of this task, in registers.
    using MW = typename XR::template MW<D>;
    constexpr int MN = XR::template MN<D>;
    MW m[NT][CPL][MN];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int c = 0; c < CPL; ++c)
            XR::template load_m<D>(M + (task * nt + (t < nt ? t : 0)) * nf, int64_t(c * S + ls) * VEC, nf, t < nt,
                                   m[t][c]);

    using AW = typename XR::template AW<D>;
    constexpr int AN = XR::template AN<D>;
    AW acc[NT][CPL][AN];  // zero bits: every element 0
    double sq = 0.0;      // LOSS: this lane's share of sum r^2
    double* wsm = smem_acc + size_t(warp) * Shape::SLOTS;
    if constexpr (GRAD) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int c = 0; c < CPL; ++c)
#pragma unroll
                for (int i = 0; i < AN; ++i) acc[t][c][i] = AW(0);
        for (int i = lane; i < Shape::SLOTS; i += kWarp) wsm[i] = 0.0;
    }

    // Fold the register partials of all row groups into the warp's double
    // accumulator (lanes of row group 0 own the shared-memory slots).
    auto flush = [&]() {
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    D val = XR::template acc_get<D>(acc[t][c], v);
                    if constexpr (!FULL) {
                        for (int off = S; off < kWarp; off <<= 1)
                            val += __shfl_xor_sync(0xffffffffu, val, off);
                    }
                    if (FULL || grp == 0) wsm[((t * CPL + c) * kWarp + ls) * VEC + v] += double(val);
                }
#pragma unroll
                for (int i = 0; i < AN; ++i) acc[t][c][i] = AW(0);
            }
    };

    // Issue the loads of one batch: U steps of R rows starting at `base`.
    // FULL batches load y only for the row whose residual this lane forms.
    // Batch-invariant parts of the addresses: this lane's vectors of a row
    // (are they inside the row?) and the distance between the batch's rows.
    bool f_ok[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) f_ok[c] = int64_t(c * S + ls) * VEC < nf;
    const T* x_lane = X + task * nf + int64_t(ls) * VEC;
    const int64_t step_elems = int64_t(R) * ntasks * nf;
    auto load = [&](XW (&xb)[U][CPL][XN], D (&yb)[U][NT], int64_t base) {
        if (base + int64_t(U - 1) * R + grp < obs_end) {
            // every row of the batch is in range (all but a CTA's last batch):
            // one pointer advanced by a row step, no per-row bounds
            const T* xrow = x_lane + (base + grp) * ntasks * nf;
#pragma unroll
            for (int u = 0; u < U; ++u) {
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    if (f_ok[c]) {
                        XR::load(xrow + c * S * VEC, xb[u][c]);
                    } else {
#pragma unroll
                        for (int v = 0; v < XN; ++v) xb[u][c][v] = XW(0);
                    }
                }
                xrow += step_elems;
            }
        } else {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t obs = base + int64_t(u) * R + grp;
                const bool ok = obs < obs_end;
                const T* xrow = x_lane + obs * ntasks * nf;
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    if (ok && f_ok[c]) {
                        XR::load(xrow + c * S * VEC, xb[u][c]);
                    } else {
#pragma unroll
                        for (int v = 0; v < XN; ++v) xb[u][c][v] = XW(0);
                    }
                }
            }
        }
        if constexpr (GRAD) {
            if constexpr (FULL) {
                const int64_t obs = base + u_mine;
                const bool ok = obs < obs_end && Y != nullptr;
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    yb[0][t] = (ok && t < nt) ? to_arith<D>(Y[(obs * ntasks + task) * nt + t]) : D(0);
            } else {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t obs = base + int64_t(u) * R + grp;
                    const bool ok = obs < obs_end && Y != nullptr;
#pragma unroll
                    for (int t = 0; t < NT; ++t)
                        yb[u][t] = (ok && t < nt) ? to_arith<D>(Y[(obs * ntasks + task) * nt + t]) : D(0);
                }
            }
        }
    };

    auto compute = [&](const XW (&xb)[U][CPL][XN], const D (&yb)[U][NT], int64_t base) {
        if constexpr (FULL) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                D vals[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    D d = D(0);
#pragma unroll
                    for (int c = 0; c < CPL; ++c) d = XR::template dot<D>(m[t][c], xb[u][c], d);
                    vals[u] = d;
                }
                // transposed butterfly over the first log2(U) lane bits
#pragma unroll
                for (int s = 0; s < LOG2U; ++s) {
                    const int o = 16 >> s;
                    const int half = U >> (s + 1);
                    const bool hi = (lane & o) != 0;
#pragma unroll
                    for (int j = 0; j < half; ++j) {
                        const D send = hi ? vals[j] : vals[j + half];
                        const D keep = hi ? vals[j + half] : vals[j];
                        vals[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                    }
                }
#pragma unroll
                for (int o = 16 >> LOG2U; o > 0; o >>= 1) vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], o);
                D d = vals[0];  // dot product of row u_mine
                if constexpr (LOGIT) d = sigmoid(d);
                if constexpr (WRITE) {
                    const int64_t obs = base + u_mine;
                    if ((lane & ((32 >> LOG2U) - 1)) == 0 && t < nt && obs < obs_end)
                        Yhat[(obs * ntasks + task) * nt + t] = T(d);
                }
                if constexpr (GRAD) {
                    const D r_mine = LOGIT ? D(0.5) * (d - yb[0][t]) : d - yb[0][t];
                    if constexpr (LOSS) {
                        const int64_t obs = base + u_mine;
                        if ((lane & ((32 >> LOG2U) - 1)) == 0 && t < nt && obs < obs_end)
                            sq = fma(double(r_mine), double(r_mine), sq);
                    }
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const auto rr = XR::template prep<D>(__shfl_sync(0xffffffffu, r_mine, u << (5 - LOG2U)));
#pragma unroll
                        for (int c = 0; c < CPL; ++c) XR::template axpy<D>(rr, xb[u][c], acc[t][c]);
                    }
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t obs = base + int64_t(u) * R + grp;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    D d = D(0);
#pragma unroll
                    for (int c = 0; c < CPL; ++c) d = XR::template dot<D>(m[t][c], xb[u][c], d);
                    for (int off = S >> 1; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
                    if constexpr (LOGIT) d = sigmoid(d);
                    if constexpr (WRITE) {
                        if (ls == 0 && t < nt && obs < obs_end) Yhat[(obs * ntasks + task) * nt + t] = T(d);
                    }
                    if constexpr (GRAD) {
                        const D r = LOGIT ? D(0.5) * (d - yb[u][t]) : d - yb[u][t];
                        if constexpr (LOSS) {
                            if (ls == 0 && t < nt && obs < obs_end) sq = fma(double(r), double(r), sq);
                        }
                        const auto rr = XR::template prep<D>(r);
#pragma unroll
                        for (int c = 0; c < CPL; ++c) XR::template axpy<D>(rr, xb[u][c], acc[t][c]);
                    }
                }
            }
        }
    };

    const int64_t warp_stride = int64_t(kRowsWarps) * U * R;
    int iters = 0;
    auto after_batch = [&]() {
        if constexpr (GRAD) {
            if (++iters == kFlushIters) {
                flush();
                iters = 0;
            }
        }
    };
    XW xa[U][CPL][XN], xb[U][CPL][XN];
    D ya[U][NT], yb[U][NT];
    int64_t base = obs_begin + int64_t(warp) * U * R;
    if (base < obs_end) load(xa, ya, base);
    while (base < obs_end) {
        int64_t next = base + warp_stride;
        if (next < obs_end) load(xb, yb, next);
        compute(xa, ya, base);
        after_batch();
        base = next;
        if (base >= obs_end) break;
        next = base + warp_stride;
        if (next < obs_end) load(xa, ya, next);
        compute(xb, yb, base);
        after_batch();
        base = next;
    }
    if constexpr (LOSS) {
        // one double per CTA: lanes, then warps, in a fixed order
        __shared__ double loss_warp[kRowsWarps];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        if (lane == 0) loss_warp[warp] = sq;
        __syncthreads();
        if (threadIdx.x == 0) {
            double s = 0.0;
#pragma unroll
            for (int w = 0; w < kRowsWarps; ++w) s += loss_warp[w];
            a.loss_part[blockIdx.x] = s;
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
            a.part[(task * K + int64_t(t) * nf + f) * a.part_stride + a.part_offset + cta] = s;
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
