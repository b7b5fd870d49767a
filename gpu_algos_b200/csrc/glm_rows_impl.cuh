// glm_rows_impl.cuh -- launch planning and dispatch of the rows kernel.
// Included by glm_rows_f16.cu / glm_rows_f32.cu / glm_rows_f64.cu, one
// instantiation per file so the element types compile in parallel.
#pragma once

#include <algorithm>

#include "glm_rows.cuh"

namespace glmb {

template <typename T>
constexpr int rows_budget() {
    // register-resident accumulator words per lane (NT * CPL * VEC): 32 for
    // float arithmetic (float and half inputs), 16 for double
    return sizeof(typename Arith<T>::Dot) == 4 ? 32 : 16;
}

template <typename T, int VEC, int CPL, int NT>
constexpr bool rows_valid() {
    return NT * CPL * VEC <= rows_budget<T>();
}

// Vectors per lane that a row shorter than a warp may take (the kernels
// instantiated for segments of fewer than 32 lanes): one, or two for float
// and double (see rows_plan).  Any longer row spans a full warp.
template <typename T, int CPL>
constexpr bool rows_short() {
    return CPL == 1 || (CPL == 2 && sizeof(T) >= 4);
}

// Calls f.template operator()<VEC, CPL, NT>() for the runtime triple.
template <typename T, typename F>
int rows_dispatch(int vec, int cpl, int ntmax, F&& f) {
    constexpr int VW = 16 / int(sizeof(T));
    auto by_nt = [&]<int VEC, int CPL>() -> int {
        switch (ntmax) {
            case 1:
                if constexpr (rows_valid<T, VEC, CPL, 1>()) return f.template operator()<VEC, CPL, 1>();
                break;
            case 2:
                if constexpr (rows_valid<T, VEC, CPL, 2>()) return f.template operator()<VEC, CPL, 2>();
                break;
            case 4:
                if constexpr (rows_valid<T, VEC, CPL, 4>()) return f.template operator()<VEC, CPL, 4>();
                break;
            case 8:
                if constexpr (rows_valid<T, VEC, CPL, 8>()) return f.template operator()<VEC, CPL, 8>();
                break;
        }
        return GLMB_ERR_UNSUPPORTED;
    };
    auto by_cpl = [&]<int VEC>() -> int {
        switch (cpl) {
            case 1: return by_nt.template operator()<VEC, 1>();
            case 2: return by_nt.template operator()<VEC, 2>();
            case 4: return by_nt.template operator()<VEC, 4>();
            case 8: return by_nt.template operator()<VEC, 8>();
        }
        return GLMB_ERR_UNSUPPORTED;
    };
    if (vec == VW) return by_cpl.template operator()<VW>();
    if (vec == 1) return by_cpl.template operator()<1>();
    if constexpr (VW == 8) {  // half: narrower vectors too (see rows_plan)
        if (vec == 4) return by_cpl.template operator()<4>();
        if (vec == 2) return by_cpl.template operator()<2>();
    }
    return GLMB_ERR_UNSUPPORTED;
}

template <typename T, int VEC, int CPL, int NT, bool FULL>
auto rows_kernel_for(int mode) {
    if (mode == kRowsGrad) return &glm_rows_kernel<T, VEC, CPL, NT, kRowsGrad, FULL>;
    if (mode == kRowsGradYhat) return &glm_rows_kernel<T, VEC, CPL, NT, kRowsGradYhat, FULL>;
    if (mode == kRowsGradLogit) return &glm_rows_kernel<T, VEC, CPL, NT, kRowsGradLogit, FULL>;
    if (mode == kRowsGradLogitYhat) return &glm_rows_kernel<T, VEC, CPL, NT, kRowsGradLogitYhat, FULL>;
    if constexpr (sizeof(T) >= 4) {  // the fused objective is offered for float and double
        if (mode == kRowsGradYhatLoss) return &glm_rows_kernel<T, VEC, CPL, NT, kRowsGradYhatLoss, FULL>;
    }
    return &glm_rows_kernel<T, VEC, CPL, NT, kRowsPredict, FULL>;
}

template <typename T, int VEC, int CPL, int NT, bool FULL>
int rows_ctas_per_sm(int mode) {
    using Shape = RowsShape<T, VEC, CPL, NT>;
    const size_t smem = mode == kRowsPredict ? 0 : Shape::SMEM;
    auto kern = rows_kernel_for<T, VEC, CPL, NT, FULL>(mode);
    // the shared-memory limit is set on every device; the occupancy is cached
    // per instance and mode (every device this library runs on is a B200)
    static std::atomic<uint64_t> attr[kRowsModes];
    if (smem > 48 * 1024) set_smem_limit_once(attr[mode], kern, smem);
    static std::atomic<int> cached[kRowsModes] = {};
    int c = cached[mode].load(std::memory_order_relaxed);
    if (c == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kRowsThreads, smem) != cudaSuccess)
            n = 1;
        c = std::max(1, n);
        cached[mode].store(c, std::memory_order_relaxed);
    }
    return c;
}

template <typename T>
RowsPlan rows_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, bool vec_aligned,
                   bool grad) {
    RowsPlan p;
    if (nf <= 0 || nt <= 0 || ntasks <= 0 || nobs < 0) return p;
    constexpr int VW = 16 / int(sizeof(T));
    p.vec = (vec_aligned && nf % VW == 0) ? VW : 1;
    if constexpr (VW == 8) {
        // half: a full warp per row with 16- or 8-byte loads (the full-warp
        // kernel reduces a batch of rows with the transposed butterfly);
        // rows too short for that take the widest vector over a narrower
        // segment.  Measured at 2^23-2^25 rows: nfeatures 128 runs 0.90 ms
        // with 8-byte loads over 32 lanes against 1.32 with 16-byte loads over
        // 16 lanes; nfeatures 64 runs 1.26 ms with 16-byte loads over 8 lanes
        // against 1.48 with 4-byte loads over 32 lanes and 2.21 with 8-byte
        // loads over 16.
        if (vec_aligned) {
            auto full = [&](int v) { return nf % v == 0 && nf / v >= kWarp; };
            int v = full(VW) ? VW : (full(VW / 2) ? VW / 2 : VW);
            while (v > 1 && nf % v != 0) v >>= 1;
            p.vec = v;
        }
    }
    const int64_t nvec = nf / p.vec;
    int cpl = 0;
    for (int c : {1, 2, 4, 8})
        if (int64_t(kWarp) * c >= nvec) {
            cpl = c;
            break;
        }
    if (cpl == 0) return p;
    int ntmax = 0;
    for (int n : {1, 2, 4, 8})
        if (n >= nt) {
            ntmax = n;
            break;
        }
    if (ntmax == 0) return p;
    if (ntmax * cpl * p.vec > rows_budget<T>()) return p;
    // Rows of 5-16 16-byte vectors (float) or 9-16 (double): two vectors per
    // lane over half the lanes (half the shuffles per row, twice the loads in
    // flight per lane).  Measured on 8-16 GiB of X: float 32 features 1.54 ms
    // against 1.82, 48 features 1.45 against 1.88, 64 features 1.50 against
    // 1.90; double 32 features 1.54 against 2.02.  Half rows are better left
    // at one vector per lane (its two-vector kernel needs 172 registers).
    if constexpr (sizeof(T) >= 4) {
        const int64_t lo = sizeof(T) == 4 ? 4 : 8;
        if (p.vec == VW && cpl == 1 && nvec > lo && nvec <= 16 && ntmax * 2 * p.vec <= rows_budget<T>()) cpl = 2;
    }
    p.cpl = cpl;
    p.ntmax = ntmax;
    const int64_t lanes = (nvec + cpl - 1) / cpl;
    int seg_log2 = 0;
    while ((int64_t(1) << seg_log2) < lanes) ++seg_log2;
    p.seg_log2 = seg_log2;
    const int mode = grad ? kRowsGrad : kRowsPredict;
    int U = 1, per_sm = 1;
    rows_dispatch<T>(p.vec, p.cpl, p.ntmax, [&]<int VEC, int CPL, int NT>() -> int {
        U = RowsShape<T, VEC, CPL, NT>::U;
        if (seg_log2 == 5) {
            per_sm = rows_ctas_per_sm<T, VEC, CPL, NT, true>(mode);
        } else if constexpr (rows_short<T, CPL>()) {
            per_sm = rows_ctas_per_sm<T, VEC, CPL, NT, false>(mode);
        }
        return GLMB_OK;
    });
    const int64_t R = kWarp >> seg_log2;
    const int64_t min_rows = int64_t(kRowsWarps) * U * R;
    const int64_t target = int64_t(sm_count()) * per_sm;
    int64_t cpt = std::max<int64_t>(1, (target + ntasks - 1) / ntasks);
    cpt = std::min<int64_t>(cpt, std::max<int64_t>(1, (nobs + min_rows - 1) / min_rows));
    int64_t opc = nobs > 0 ? (nobs + cpt - 1) / cpt : 1;
    opc = (opc + R - 1) / R * R;
    cpt = nobs > 0 ? (nobs + opc - 1) / opc : 0;
    if (cpt * ntasks > int64_t(0x7fffffff)) return p;
    p.ctas_per_task = int32_t(cpt);
    p.obs_per_cta = opc;
    p.part_doubles = size_t(ntasks) * size_t(nt) * size_t(nf) * size_t(cpt);
    p.ok = true;
    return p;
}

template <typename T>
int rows_launch(const RowsPlan& p, int mode, const RowsArgs& args, cudaStream_t stream) {
    if (mode < 0 || mode >= kRowsModes) return GLMB_ERR_INVALID_VALUE;
    if (mode == kRowsGradYhatLoss && sizeof(T) < 4) return GLMB_ERR_UNSUPPORTED;
    if (p.ctas_per_task == 0) return GLMB_OK;  // no observations: nothing to launch
    if (mode == kRowsGradYhatLoss && args.loss_part == nullptr) return GLMB_ERR_INVALID_VALUE;
    return rows_dispatch<T>(p.vec, p.cpl, p.ntmax, [&]<int VEC, int CPL, int NT>() -> int {
        using Shape = RowsShape<T, VEC, CPL, NT>;
        const size_t smem = mode == kRowsPredict ? 0 : Shape::SMEM;
        const dim3 grid(unsigned(int64_t(p.ctas_per_task) * args.ntasks));
        if (p.seg_log2 == 5) {
            rows_ctas_per_sm<T, VEC, CPL, NT, true>(mode);  // sets the shared-memory attribute once
            rows_kernel_for<T, VEC, CPL, NT, true>(mode)<<<grid, kRowsThreads, smem, stream>>>(args);
        } else {
            if constexpr (rows_short<T, CPL>()) {
                rows_ctas_per_sm<T, VEC, CPL, NT, false>(mode);
                rows_kernel_for<T, VEC, CPL, NT, false>(mode)<<<grid, kRowsThreads, smem, stream>>>(args);
            } else {
                return GLMB_ERR_UNSUPPORTED;  // rows_plan never makes such a plan
            }
        }
        count_launch();
        return launch_status();
    });
}

#define GLMB_INSTANTIATE_ROWS(T)                                                              \
    template RowsPlan rows_plan<T>(int64_t, int64_t, int64_t, int64_t, bool, bool);          \
    template int rows_launch<T>(const RowsPlan&, int, const RowsArgs&, cudaStream_t);

}  // namespace glmb
