// glm_noalloc.cu -- a float32 gradient entry point that allocates no device memory.
//
// glmb_gradient_f32 needs a little scratch (one double per task x target x
// feature x CTA) and, when the caller passes none, takes it with
// cudaMallocAsync.  Some callers cannot let a library allocate: a host
// application that owns every device buffer itself and hands a plugin only
// its inputs and outputs (the reference's driver is built that way), code
// whose device-memory budget is fixed once at start-up, or a latency-critical
// path that must not wait on the allocator.  glmb_gradient_noalloc_f32 serves
// them: its scratch is the file-scope device array below, sized once for the
// largest problem it accepts.
//
// Rules of use (also stated in include/glm_b200.h):
//  - The array is 4 MiB (kNoAllocScratchDoubles doubles) and lives on every
//    GPU that loads this library until the process exits.
//  - It holds one double per (task, target, feature) per CTA, so the call
//    rejects nfeatures*ntargets*ntasks > kNoAllocScratchDoubles with
//    GLMB_ERR_TOO_LARGE; below that it lowers the CTA count if needed.
//  - Only shapes served by the single-pass kernel are accepted (ntargets <= 8,
//    nfeatures up to 1024); others return GLMB_ERR_UNSUPPORTED.
//  - Every call on a device shares the one array, which keeps the previous
//    call's contents.  Nothing in it needs to start at zero: each slot a call
//    reads is written earlier in the same call.  Two calls whose kernels
//    overlap on the GPU (different streams, no ordering between them) race on
//    the array and corrupt each other's result; order them on one stream or
//    with events.
//  - The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture begins.  The cached address lives
//    as long as the process: after cudaDeviceReset on a device, this entry
//    point must not be called again in that process (the module would be
//    reloaded and the array could move).
//  - When the array, not the GPU, limits the CTAs a task gets (fewer than the
//    planner's 148 SMs x CTAs per SM), each CTA walks more rows and the call
//    slows in proportion.
#include <mutex>

#include "glm_common.cuh"
#include "glm_generic.cuh"
#include "glm_rows.cuh"

namespace {

constexpr size_t kNoAllocScratchDoubles = size_t(1) << 19;  // 4 MiB

}  // namespace

// Host code must not take this symbol's address as a device pointer: on the
// host it names a stand-in object.  The device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) double g_noalloc_scratch[kNoAllocScratchDoubles];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
double* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (set up once).
int noalloc_scratch(double** out, int* major) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return int(e);
    if (dev < 0 || dev >= kMaxDevices) return GLMB_ERR_UNSUPPORTED;
    if ((e = cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
        return int(e);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return int(e);
        g_noalloc_ptr[dev] = static_cast<double*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return GLMB_OK;
}

int gradient_noalloc(const float* X, const float* M, const float* Y, float* grad, float* Yhat,
                     int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, double lambda,
                     double alpha, uint32_t flags, cudaStream_t stream) {
    using namespace glmb;
    if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0) return GLMB_ERR_INVALID_VALUE;
    if (flags & ~(GLMB_GRAD_REGULARIZE | GLMB_GRAD_WRITE_YHAT | GLMB_GRAD_Y_ZERO))
        return GLMB_ERR_INVALID_VALUE;
    const bool reg = (flags & GLMB_GRAD_REGULARIZE) != 0;
    const bool write_yhat = (flags & GLMB_GRAD_WRITE_YHAT) != 0;
    const bool y_zero = (flags & GLMB_GRAD_Y_ZERO) != 0;
    if (nt == 0 || ntasks == 0) return GLMB_OK;
    const int64_t nout = nobs * ntasks * nt;
    if (write_yhat && nout > 0 && Yhat == nullptr) return GLMB_ERR_INVALID_VALUE;
    const int64_t K = nf * nt * ntasks;
    if (K > int64_t(kNoAllocScratchDoubles)) return GLMB_ERR_TOO_LARGE;
    double* scratch = nullptr;
    int major = 0;
    int st = noalloc_scratch(&scratch, &major);
    if (st != GLMB_OK) return st;
    if (major != 10) return GLMB_ERR_UNSUPPORTED;
    if (nf == 0) {
        if (write_yhat && nout > 0) return int(cudaMemsetAsync(Yhat, 0, size_t(nout) * sizeof(float), stream));
        return GLMB_OK;
    }
    if (M == nullptr || grad == nullptr) return GLMB_ERR_INVALID_VALUE;
    if (nobs > 0 && (X == nullptr || (!y_zero && Y == nullptr))) return GLMB_ERR_INVALID_VALUE;
    const bool aligned = (reinterpret_cast<uintptr_t>(X) & 15u) == 0;
    RowsPlan p = rows_plan<float>(nf, nt, ntasks, nobs, aligned, true);
    if (!p.ok) return GLMB_ERR_UNSUPPORTED;
    // fit the CTA partials into the fixed array: fewer, longer CTAs if needed
    const int64_t cpt_max = int64_t(kNoAllocScratchDoubles) / K;
    if (int64_t(p.ctas_per_task) > cpt_max) {
        const int64_t R = int64_t(kWarp) >> p.seg_log2;
        int64_t opc = (nobs + cpt_max - 1) / cpt_max;
        opc = (opc + R - 1) / R * R;
        p.obs_per_cta = opc;
        p.ctas_per_task = int32_t((nobs + opc - 1) / opc);
        p.part_doubles = size_t(K) * size_t(p.ctas_per_task);
    }
    RowsArgs a{X, M, y_zero ? nullptr : Y, write_yhat ? Yhat : nullptr, scratch, nf, nt, ntasks, nobs,
               p.obs_per_cta, p.ctas_per_task, 0, p.ctas_per_task, p.seg_log2};
    st = rows_launch<float>(p, write_yhat ? kRowsGradYhat : kRowsGrad, a, stream);
    if (st != GLMB_OK) return st;
    return finalize_launch<float, double>(scratch, p.ctas_per_task, K, M, grad, nullptr, lambda, alpha,
                                          reg, stream);
}

}  // namespace

extern "C" int glmb_gradient_noalloc_f32(const float* X, const float* M, const float* Y, float* grad_M,
                                         float* Yhat, int64_t nfeatures, int64_t ntargets,
                                         int64_t ntasks, int64_t nobs, double lambda, double alpha,
                                         uint32_t flags, glmb_stream_t stream) {
    try {
        return gradient_noalloc(X, M, Y, grad_M, Yhat, nfeatures, ntargets, ntasks, nobs, lambda, alpha,
                                flags, reinterpret_cast<cudaStream_t>(stream));
    } catch (...) {
        return GLMB_ERR_INVALID_VALUE;
    }
}
