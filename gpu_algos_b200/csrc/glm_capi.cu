// glm_capi.cu -- the extern "C" entry points declared in include/glm_b200.h.
//
// Each entry point validates its arguments, picks a kernel family and
// launches asynchronously on the caller's stream:
//   - "rows":    fused single-pass kernel (glm_rows.cuh) for half/float/
//                double when ntargets <= 8 and the per-lane accumulators fit
//                in registers (with a single target and 16-byte-aligned
//                rows nfeatures up to 1024 for half and float, 512 for
//                double; 256 with unaligned rows);
//   - "tiles":   float64 with up to 16 targets and 256 features that the
//                rows kernel cannot hold in registers: shared-memory tiles
//                filled by cp.async.bulk, both contractions on the FP64
//                tensor pipe (glm_tiles.cu);
//   - "dense":   float32 shapes the rows kernel cannot hold (many targets
//                or features): two TMA-fed tcgen05 GEMMs with 3xTF32
//                precision (glm_dense.cu);
//   - "generic": two-pass kernels (glm_generic.cu) for every other shape and
//                for half and integer types.
// Nothing here falls back to the host: a missing or failing device returns
// the CUDA error code.
#include <cstring>
#include <mutex>

#include "glm_common.cuh"
#include "glm_dense.cuh"
#include "glm_loss.cuh"
#include "glm_fit.cuh"
#include "glm_generic.cuh"
#include "glm_peer.cuh"
#include "glm_rows.cuh"
#include "glm_tiles.cuh"

namespace glmb {

namespace {
std::atomic<uint64_t> g_launches{0};
thread_local const char* g_last_path = "none";

struct DeviceInfo {
    int sm = 0;
    int major = 0;
};
DeviceInfo g_devices[64];
std::mutex g_dev_mutex;

int device_info(DeviceInfo* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return int(e);
    if (dev < 0 || dev >= 64) return GLMB_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    DeviceInfo& d = g_devices[dev];
    if (d.sm == 0) {
        if ((e = cudaDeviceGetAttribute(&d.sm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return int(e);
        if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return int(e);
    }
    *out = d;
    return GLMB_OK;
}
}  // namespace

void count_launch(int n) { g_launches.fetch_add(uint64_t(n), std::memory_order_relaxed); }
void set_last_path(const char* path) { g_last_path = path; }

int sm_count() {
    DeviceInfo d;
    return device_info(&d) == GLMB_OK && d.sm > 0 ? d.sm : 148;
}

namespace {

// The library carries sm_100a code only.
int check_device() {
    DeviceInfo d;
    const int st = device_info(&d);
    if (st != GLMB_OK) return st;
    return d.major == 10 ? GLMB_OK : GLMB_ERR_UNSUPPORTED;
}

template <typename T>
constexpr bool kRowsType = std::is_same_v<T, float> || std::is_same_v<T, double>;
// element types the fused rows kernel is built for (half, bfloat16: float arithmetic on packed 4- to
// 16-byte loads)
template <typename T>
constexpr bool kRowsKernelType = kRowsType<T> || kHalf16<T>;
// element types with the peer exchange (glmb_gradient_sharded_*)
template <typename T>
constexpr bool kPeerType = kRowsType<T> || kHalf16<T>;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
int predict_impl(const T* X, const T* M, T* Yhat, int64_t nf, int64_t nt, int64_t ntasks,
                 int64_t nobs, cudaStream_t stream) {
    if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0) return GLMB_ERR_INVALID_VALUE;
    const int64_t nout = nt * ntasks * nobs;
    if (nout == 0) return GLMB_OK;
    if (Yhat == nullptr) return GLMB_ERR_INVALID_VALUE;
    int st = check_device();
    if (st != GLMB_OK) return st;
    if (nf == 0) {
        set_last_path("memset");
        return int(cudaMemsetAsync(Yhat, 0, size_t(nout) * sizeof(T), stream));
    }
    if (X == nullptr || M == nullptr) return GLMB_ERR_INVALID_VALUE;
    if constexpr (kRowsKernelType<T>) {
        const RowsPlan p = rows_plan<T>(nf, nt, ntasks, nobs, aligned16(X), false);
        if (p.ok) {
            RowsArgs a{X, M, nullptr, Yhat, nullptr, nf, nt, ntasks, nobs, p.obs_per_cta,
                       p.ctas_per_task, 0, p.ctas_per_task, p.seg_log2};
            set_last_path("rows");
            return rows_launch<T>(p, kRowsPredict, a, stream);
        }
    }
    set_last_path("generic");
    return generic_predict<T>(X, M, Yhat, nf, nt, ntasks, nobs, stream);
}

template <typename T>
size_t gradient_ws_impl(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {
    if (nf <= 0 || nt <= 0 || ntasks <= 0 || nobs < 0) return 0;
    if (check_device() != GLMB_OK) return 0;
    size_t need = 0;
    bool all_rows = false;
    if constexpr (kRowsKernelType<T>) {
        const RowsPlan a = rows_plan<T>(nf, nt, ntasks, nobs, true, true);
        const RowsPlan b = rows_plan<T>(nf, nt, ntasks, nobs, false, true);
        all_rows = a.ok && b.ok;
        // the CTA partials, then (glmb_gradient_loss_*) one squared-residual sum per CTA
        auto rows_need = [&](const RowsPlan& p) {
            return round_up(p.part_doubles * sizeof(double), 256) +
                   round_up(size_t(ntasks) * size_t(p.ctas_per_task) * sizeof(double), 256);
        };
        if (a.ok) need = std::max(need, rows_need(a));
        if (b.ok) need = std::max(need, rows_need(b));
    }
    if constexpr (std::is_same_v<T, float>) {
        if (!all_rows && dense_f32_supported(nf, nt, ntasks, std::max<int64_t>(nobs, 1), nullptr, nullptr)) {
            const DensePlan dp = dense_f32_plan(nf, nt, ntasks, std::max<int64_t>(nobs, 1));
            need = std::max(need, dp.ws_bytes + round_up(size_t(ntasks) * nt * nf * sizeof(double), 256));
        }
    }
    if constexpr (std::is_same_v<T, double>) {
        if (!all_rows && tiles_f64_supported(nf, nt, ntasks, nullptr)) {
            const TilesPlan tp = tiles_f64_plan(nf, nt, ntasks, nobs);
            need = std::max(need, round_up(tp.part_doubles * sizeof(double), 256) + 256);
        }
    }
    if (!all_rows) need = std::max(need, generic_workspace_bytes<T>(nf, nt, ntasks, nobs));
    // glmb_gradient_loss_* reuses the workspace for the loss after the gradient
    return std::max(need, loss_workspace_bytes());
}

// Shared body of glmb_gradient_* (partial_out == NULL) and
// glmb_gradient_partial_* (partial_out != NULL, grad unused).
template <typename T>
struct PeerFinish {
    glmb_peer_group* g;
    const T* M;
    T* grad;
    double* partial_out;
    double lambda, alpha;
    bool reg;
    const int* local_status;
    int64_t total;
    cudaStream_t stream;
    static int call(void* ctx, const void* part, int64_t nparts) {
        auto* f = static_cast<PeerFinish*>(ctx);
        return exchange_launch<T>(f->g, static_cast<const double*>(part), nparts, f->total, f->M, f->grad,
                                  f->partial_out, f->lambda, f->alpha, f->reg, f->local_status, f->stream);
    }
};

// With `peer` set (float/double only), the CTA partials are summed across
// the ranks of the group by the exchange kernel instead of the local finalize.
// With `fused_loss` set (float/double, Yhat written, one GPU), a shape that
// the rows kernel serves also gets the objective in fused_loss[0] from the
// same pass over X, Y and M, and *loss_done says so; other shapes leave the
// loss to the caller.
template <typename T>
int gradient_impl(const T* X, const T* M, const T* Y, T* grad, T* Yhat, double* partial_out,
                  int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, double lambda, double alpha,
                  uint32_t flags, void* ws, size_t ws_bytes, cudaStream_t stream,
                  glmb_peer_group* peer = nullptr, T* fused_loss = nullptr, bool* loss_done = nullptr) {
    if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0) return GLMB_ERR_INVALID_VALUE;
    if (flags & ~(GLMB_GRAD_REGULARIZE | GLMB_GRAD_WRITE_YHAT | GLMB_GRAD_Y_ZERO | GLMB_GRAD_LOGISTIC))
        return GLMB_ERR_INVALID_VALUE;
    const bool logistic = (flags & GLMB_GRAD_LOGISTIC) != 0;
    if (logistic && !std::is_floating_point_v<T> && !kHalf16<T>) return GLMB_ERR_INVALID_VALUE;
    if (peer != nullptr && !kPeerType<T>) return GLMB_ERR_UNSUPPORTED;
    const bool reg = (flags & GLMB_GRAD_REGULARIZE) != 0;
    const bool write_yhat = (flags & GLMB_GRAD_WRITE_YHAT) != 0;
    const bool y_zero = (flags & GLMB_GRAD_Y_ZERO) != 0;
    if (nt == 0 || ntasks == 0) return GLMB_OK;
    const int64_t nout = nobs * ntasks * nt;
    if (write_yhat && nout > 0 && Yhat == nullptr) return GLMB_ERR_INVALID_VALUE;
    int st = check_device();
    if (st != GLMB_OK) return st;
    if (nf == 0 && !logistic) {
        set_last_path("memset");
        if (write_yhat && nout > 0)
            return int(cudaMemsetAsync(Yhat, 0, size_t(nout) * sizeof(T), stream));
        return GLMB_OK;
    }
    if (M == nullptr || (partial_out == nullptr && grad == nullptr)) return GLMB_ERR_INVALID_VALUE;
    if (nobs > 0 && (X == nullptr || (!y_zero && Y == nullptr))) return GLMB_ERR_INVALID_VALUE;
    const T* Yin = y_zero ? nullptr : Y;
    T* Yhat_out = write_yhat ? Yhat : nullptr;
    if constexpr (kRowsKernelType<T>) {
        const RowsPlan p = rows_plan<T>(nf, nt, ntasks, nobs, aligned16(X), true);
        if (p.ok) {
            const bool fuse = kRowsType<T> && fused_loss != nullptr && loss_done != nullptr && write_yhat &&
                              !logistic && peer == nullptr && partial_out == nullptr;
            const size_t part_bytes = round_up(p.part_doubles * sizeof(double), 256);
            const int64_t nloss = ntasks * int64_t(p.ctas_per_task);
            Scratch sc(ws, ws_bytes, part_bytes + (fuse ? round_up(size_t(nloss) * sizeof(double), 256) : 0),
                       stream);
            if (sc.status() != GLMB_OK) return sc.status();
            double* loss_part = fuse ? reinterpret_cast<double*>(sc.as<char>() + part_bytes) : nullptr;
            RowsArgs a{X, M, Yin, Yhat_out, sc.as<double>(), nf, nt, ntasks, nobs, p.obs_per_cta,
                       p.ctas_per_task, 0, p.ctas_per_task, p.seg_log2, loss_part};
            set_last_path("rows");
            const int mode = logistic ? (write_yhat ? kRowsGradLogitYhat : kRowsGradLogit)
                                      : (fuse ? kRowsGradYhatLoss : (write_yhat ? kRowsGradYhat : kRowsGrad));
            st = rows_launch<T>(p, mode, a, stream);
            if (st != GLMB_OK) return st;
            if constexpr (kRowsType<T>) {
                if (fuse) {
                    st = finalize_launch<T, double>(sc.as<double>(), p.ctas_per_task, ntasks * nt * nf, M, grad,
                                                    nullptr, lambda, alpha, reg, stream);
                    if (st != GLMB_OK) return st;
                    *loss_done = true;
                    return loss_from_partials_launch<T>(loss_part, nloss, M, ntasks * nt * nf, fused_loss, lambda,
                                                        alpha, stream);
                }
            }
            if constexpr (kPeerType<T>) {
                if (peer != nullptr)
                    return exchange_launch<T>(peer, sc.as<double>(), p.ctas_per_task, ntasks * nt * nf, M, grad,
                                              partial_out, lambda, alpha, reg, nullptr, stream);
            }
            return finalize_launch<T, double>(sc.as<double>(), p.ctas_per_task, ntasks * nt * nf, M,
                                              grad, partial_out, lambda, alpha, reg, stream);
        }
    }
    if constexpr (std::is_same_v<T, float>) {
        if (!logistic && nobs > 0 && dense_f32_supported(nf, nt, ntasks, nobs, X, M)) {
            const DensePlan dp = dense_f32_plan(nf, nt, ntasks, nobs);
            const int64_t total = ntasks * nt * nf;
            const size_t local_bytes = peer != nullptr ? round_up(size_t(total) * sizeof(double), 256) : 0;
            Scratch sc(ws, ws_bytes, dp.ws_bytes + local_bytes, stream);
            if (sc.status() != GLMB_OK) return sc.status();
            set_last_path("dense");
            if (peer == nullptr)
                return dense_f32_gradient(dp, X, M, Yin, grad, Yhat_out, partial_out, nf, nt, ntasks, nobs, lambda,
                                          alpha, reg, sc.as<void>(), stream);
            double* local = reinterpret_cast<double*>(sc.as<char>() + dp.ws_bytes);
            st = dense_f32_gradient(dp, X, M, Yin, nullptr, Yhat_out, local, nf, nt, ntasks, nobs, 0.0, 0.0, false,
                                    sc.as<void>(), stream);
            if (st != GLMB_OK) return st;
            return exchange_launch<T>(peer, local, 1, total, M, grad, partial_out, lambda, alpha, reg, nullptr,
                                      stream);
        }
    }
    if constexpr (std::is_same_v<T, double>) {
        if (!logistic && tiles_f64_supported(nf, nt, ntasks, X)) {
            const TilesPlan tp = tiles_f64_plan(nf, nt, ntasks, nobs);
            const size_t part_bytes = round_up(tp.part_doubles * sizeof(double), 256);
            Scratch sc(ws, ws_bytes, part_bytes + 256, stream);
            if (sc.status() != GLMB_OK) return sc.status();
            double* part = sc.as<double>();
            int* status = reinterpret_cast<int*>(sc.as<char>() + part_bytes);
            cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream);
            if (e != cudaSuccess) return int(e);
            set_last_path("tiles");
            st = tiles_f64_launch(tp, X, M, Yin, Yhat_out, part, status, nf, nt, ntasks, nobs, stream);
            if (st != GLMB_OK) return st;
            if (peer != nullptr)
                return exchange_launch<T>(peer, part, tp.ctas_per_task, ntasks * nt * nf, M, grad, partial_out,
                                          lambda, alpha, reg, status, stream);
            st = finalize_launch<T, double>(part, tp.ctas_per_task, ntasks * nt * nf, M, grad, partial_out,
                                            lambda, alpha, reg, stream);
            if (st != GLMB_OK) return st;
            return tiles_poison(status, partial_out, partial_out ? nullptr : grad, ntasks * nt * nf, stream);
        }
    }
    set_last_path("generic");
    if constexpr (kPeerType<T>) {
        if (peer != nullptr) {
            PeerFinish<T> fin{peer, M, grad, partial_out, lambda, alpha, reg, nullptr, ntasks * nt * nf, stream};
            return generic_gradient<T>(X, M, Yin, grad, Yhat_out, partial_out, nf, nt, ntasks, nobs, lambda,
                                       alpha, reg, ws, ws_bytes, stream, &PeerFinish<T>::call, &fin, logistic);
        }
    }
    return generic_gradient<T>(X, M, Yin, grad, Yhat_out, partial_out, nf, nt, ntasks, nobs, lambda,
                               alpha, reg, ws, ws_bytes, stream, nullptr, nullptr, logistic);
}

template <typename T>
size_t fit_ws_impl(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {
    const size_t grad_ws = std::max(gradient_ws_impl<T>(nf, nt, ntasks, nobs),
                                    gradient_ws_impl<T>(nf, 1, ntasks, nobs));
    const size_t part = round_up(size_t(ntasks) * std::max<int64_t>(nt, 1) * nf * sizeof(double), 256);
    const size_t v = round_up(size_t(ntasks) * nf * sizeof(T), 256);
    const size_t norm = round_up(size_t(ntasks) * sizeof(double), 256);
    return grad_ws + part + v + norm;
}

// The whole fit on one GPU, or -- with `group` -- on this rank's block of
// observations, every partial sum completed over the group's ranks by the
// exchange kernel (so every rank holds the same L and beta throughout).
template <typename T>
int fit_impl(const T* X, const T* Y, T* beta, double* lipschitz, int64_t nf, int64_t nt,
             int64_t ntasks, int64_t nobs, double lambda1, double lambda2, int n_power, int n_iter,
             uint64_t seed, void* ws, size_t ws_bytes, cudaStream_t stream, glmb_peer_group* group = nullptr) {
    if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0 || n_power < 0 || n_iter < 0)
        return GLMB_ERR_INVALID_VALUE;
    if (lambda1 < 0 || lambda2 < 0) return GLMB_ERR_INVALID_VALUE;
    if (nf == 0 || nt == 0 || ntasks == 0) return GLMB_OK;
    if (beta == nullptr || lipschitz == nullptr) return GLMB_ERR_INVALID_VALUE;
    if (n_iter > 0 && n_power < 1) return GLMB_ERR_INVALID_VALUE;
    int st = check_device();
    if (st != GLMB_OK) return st;
    const size_t grad_ws = std::max(gradient_ws_impl<T>(nf, nt, ntasks, nobs),
                                    gradient_ws_impl<T>(nf, 1, ntasks, nobs));
    Scratch sc(ws, ws_bytes, fit_ws_impl<T>(nf, nt, ntasks, nobs), stream);
    if (sc.status() != GLMB_OK) return sc.status();
    char* base = sc.as<char>();
    void* gws = base;
    double* part = reinterpret_cast<double*>(base + grad_ws);
    T* v = reinterpret_cast<T*>(base + grad_ws +
                                round_up(size_t(ntasks) * nt * nf * sizeof(double), 256));
    double* norm = reinterpret_cast<double*>(reinterpret_cast<char*>(v) +
                                             round_up(size_t(ntasks) * nf * sizeof(T), 256));
    const int64_t K = nt * nf;
    if ((st = power_init<T>(v, nf, ntasks, seed, stream)) != GLMB_OK) return st;
    for (int it = 0; it < n_power; ++it) {
        st = gradient_impl<T>(X, v, nullptr, nullptr, nullptr, part, nf, 1, ntasks, nobs, 0.0, 0.0,
                              GLMB_GRAD_Y_ZERO, gws, grad_ws, stream, group);
        if (st != GLMB_OK) return st;
        if ((st = power_step<T>(part, v, norm, lipschitz, nf, ntasks, lambda2, stream)) != GLMB_OK)
            return st;
    }
    cudaError_t e = cudaMemsetAsync(beta, 0, size_t(K * ntasks) * sizeof(T), stream);
    if (e != cudaSuccess) return int(e);
    for (int it = 0; it < n_iter; ++it) {
        st = gradient_impl<T>(X, beta, Y, nullptr, nullptr, part, nf, nt, ntasks, nobs, 0.0, 0.0, 0u,
                              gws, grad_ws, stream, group);
        if (st != GLMB_OK) return st;
        if ((st = prox_update<T>(part, beta, lipschitz, K, ntasks, lambda1, lambda2, stream)) != GLMB_OK)
            return st;
    }
    return GLMB_OK;
}

// Exceptions (std::bad_alloc from the standard library) never cross the ABI.
template <typename F>
int guarded(F&& f) {
    try {
        return f();
    } catch (...) {
        return GLMB_ERR_INVALID_VALUE;
    }
}

}  // namespace

// Entry points for the single-process multi-GPU context (glm_mg.cu).
template <typename T>
int sharded_gradient(const T* X, const T* M, const T* Y, T* grad, double* partial_out, int64_t nf, int64_t nt,
                     int64_t ntasks, int64_t nobs, double lambda, double alpha, uint32_t flags,
                     cudaStream_t stream, glmb_peer_group* group) {
    return guarded([&] {
        return gradient_impl<T>(X, M, Y, partial_out ? nullptr : grad, nullptr, partial_out, nf, nt, ntasks, nobs,
                                lambda, alpha, flags, nullptr, 0, stream, group);
    });
}
template int sharded_gradient<float>(const float*, const float*, const float*, float*, double*, int64_t, int64_t,
                                     int64_t, int64_t, double, double, uint32_t, cudaStream_t, glmb_peer_group*);
template int sharded_gradient<double>(const double*, const double*, const double*, double*, double*, int64_t,
                                      int64_t, int64_t, int64_t, double, double, uint32_t, cudaStream_t,
                                      glmb_peer_group*);
int device_check() { return check_device(); }

}  // namespace glmb

using glmb::guarded;

extern "C" {

int glmb_version(void) { return 100; }

const char* glmb_status_string(int status) {
    switch (status) {
        case GLMB_OK: return "success";
        case GLMB_ERR_INVALID_VALUE: return "invalid argument (negative size or NULL pointer)";
        case GLMB_ERR_WORKSPACE: return "workspace smaller than required";
        case GLMB_ERR_UNSUPPORTED:
            return "unsupported: no sm_100 device (libglm_b200 carries sm_100a code only), or options this entry "
                   "point does not offer";
        case GLMB_ERR_TOO_LARGE: return "size beyond a documented limit";
        case GLMB_ERR_COLLECTIVE: return "NCCL could not be loaded, or an NCCL call failed";
        case GLMB_ERR_PEER_TIMEOUT: return "a wait for a peer's partial ran out (that call's outputs are NaN)";
        default:
            if (status > 0 && status < 1000) return cudaGetErrorString(static_cast<cudaError_t>(status));
            return "unknown status";
    }
}

uint64_t glmb_launch_count(void) { return glmb::g_launches.load(std::memory_order_relaxed); }

const char* glmb_last_path(void) { return glmb::g_last_path; }

#define GLMB_DEFINE_BASIC(SFX, CT, NT_)                                                            \
    int glmb_predict_##SFX(const CT* X, const CT* M, CT* Yhat, int64_t nf, int64_t nt,            \
                           int64_t ntasks, int64_t nobs, glmb_stream_t stream) {                   \
        return guarded([&] {                                                                       \
            return glmb::predict_impl<NT_>(reinterpret_cast<const NT_*>(X),                        \
                                           reinterpret_cast<const NT_*>(M),                        \
                                           reinterpret_cast<NT_*>(Yhat), nf, nt, ntasks, nobs,     \
                                           reinterpret_cast<cudaStream_t>(stream));                \
        });                                                                                        \
    }                                                                                              \
    size_t glmb_gradient_workspace_size_##SFX(int64_t nf, int64_t nt, int64_t ntasks,             \
                                              int64_t nobs) {                                      \
        try {                                                                                      \
            return glmb::gradient_ws_impl<NT_>(nf, nt, ntasks, nobs);                              \
        } catch (...) {                                                                            \
            return 0;                                                                              \
        }                                                                                          \
    }                                                                                              \
    int glmb_gradient_##SFX(const CT* X, const CT* M, const CT* Y, CT* grad_M, CT* Yhat,          \
                            int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, double lambda,   \
                            double alpha, uint32_t flags, void* workspace, size_t workspace_bytes, \
                            glmb_stream_t stream) {                                                \
        return guarded([&] {                                                                       \
            return glmb::gradient_impl<NT_>(                                                       \
                reinterpret_cast<const NT_*>(X), reinterpret_cast<const NT_*>(M),                  \
                reinterpret_cast<const NT_*>(Y), reinterpret_cast<NT_*>(grad_M),                   \
                reinterpret_cast<NT_*>(Yhat), nullptr, nf, nt, ntasks, nobs, lambda, alpha, flags, \
                workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));               \
        });                                                                                        \
    }                                                                                              \
    int glmb_loss_##SFX(const CT* M, const CT* Y, const CT* Yhat, CT* loss, int64_t nf, int64_t nt, \
                        int64_t ntasks, int64_t nobs, double lambda, double alpha, void* workspace, \
                        size_t workspace_bytes, glmb_stream_t stream) {                            \
        if (nf < 0 || nt < 0 || ntasks < 0 || nobs < 0) return GLMB_ERR_INVALID_VALUE;             \
        return guarded([&] {                                                                       \
            const int st = glmb::check_device();                                                   \
            if (st != GLMB_OK) return st;                                                          \
            return glmb::loss_launch<NT_>(                                                         \
                reinterpret_cast<const NT_*>(M), reinterpret_cast<const NT_*>(Y),                  \
                reinterpret_cast<const NT_*>(Yhat), reinterpret_cast<NT_*>(loss), nf, nt, ntasks,  \
                nobs, lambda, alpha, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream)); \
        });                                                                                        \
    }

GLMB_DEFINE_BASIC(f16, uint16_t, __half)
GLMB_DEFINE_BASIC(bf16, uint16_t, __nv_bfloat16)
GLMB_DEFINE_BASIC(f32, float, float)
GLMB_DEFINE_BASIC(f64, double, double)
GLMB_DEFINE_BASIC(i8, int8_t, int8_t)
GLMB_DEFINE_BASIC(i16, int16_t, int16_t)
GLMB_DEFINE_BASIC(i32, int32_t, int32_t)
GLMB_DEFINE_BASIC(i64, int64_t, int64_t)
GLMB_DEFINE_BASIC(u8, uint8_t, uint8_t)
GLMB_DEFINE_BASIC(u16, uint16_t, uint16_t)
GLMB_DEFINE_BASIC(u32, uint32_t, uint32_t)
GLMB_DEFINE_BASIC(u64, uint64_t, uint64_t)

#define GLMB_DEFINE_FLOATING(SFX, T)                                                               \
    int glmb_gradient_loss_##SFX(const T* X, const T* M, const T* Y, T* grad_M, T* Yhat, T* loss,  \
                                 int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,             \
                                 double lambda, double alpha, uint32_t flags, void* workspace,     \
                                 size_t workspace_bytes, glmb_stream_t stream) {                   \
        if (loss == nullptr || (Yhat == nullptr && nobs * nt * ntasks > 0)) return GLMB_ERR_INVALID_VALUE; \
        if (flags & GLMB_GRAD_LOGISTIC) return GLMB_ERR_UNSUPPORTED; /* the loss is the squared error */ \
        return guarded([&] {                                                                       \
            const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);                         \
            bool fused = false; /* the rows kernel summed the squared residuals */                 \
            int st = glmb::gradient_impl<T>(X, M, Y, grad_M, Yhat, nullptr, nf, nt, ntasks, nobs,  \
                                            lambda, alpha, flags | GLMB_GRAD_WRITE_YHAT, workspace, \
                                            workspace_bytes, s, nullptr, loss, &fused);            \
            if (st != GLMB_OK || fused) return st;                                                 \
            /* the gradient's scratch is free again in stream order */                             \
            return glmb::loss_launch<T>(M, (flags & GLMB_GRAD_Y_ZERO) ? nullptr : Y, Yhat, loss, nf, nt, \
                                        ntasks, nobs, lambda, alpha, workspace, workspace_bytes, s); \
        });                                                                                        \
    }                                                                                              \
    int glmb_gradient_partial_##SFX(const T* X, const T* M, const T* Y, double* partial, T* Yhat, \
                                    int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,          \
                                    uint32_t flags, void* workspace, size_t workspace_bytes,       \
                                    glmb_stream_t stream) {                                        \
        if (partial == nullptr && nf > 0 && nt > 0 && ntasks > 0) return GLMB_ERR_INVALID_VALUE;   \
        return guarded([&] {                                                                       \
            return glmb::gradient_impl<T>(X, M, Y, nullptr, Yhat, partial, nf, nt, ntasks, nobs,   \
                                          0.0, 0.0, flags & ~GLMB_GRAD_REGULARIZE, workspace,      \
                                          workspace_bytes, reinterpret_cast<cudaStream_t>(stream)); \
        });                                                                                        \
    }                                                                                              \
    int glmb_gradient_finalize_##SFX(const double* partial, const T* M, T* grad_M, int64_t nf,    \
                                     int64_t nt, int64_t ntasks, double lambda, double alpha,      \
                                     uint32_t flags, glmb_stream_t stream) {                       \
        if (nf < 0 || nt < 0 || ntasks < 0) return GLMB_ERR_INVALID_VALUE;                         \
        const int64_t total = nf * nt * ntasks;                                                    \
        if (total == 0) return GLMB_OK;                                                            \
        if (partial == nullptr || M == nullptr || grad_M == nullptr) return GLMB_ERR_INVALID_VALUE; \
        return guarded([&] {                                                                       \
            const int st = glmb::check_device();                                                   \
            if (st != GLMB_OK) return st;                                                          \
            return glmb::finalize_launch<T, double>(partial, 1, total, M, grad_M, nullptr, lambda, \
                                                    alpha, (flags & GLMB_GRAD_REGULARIZE) != 0,    \
                                                    reinterpret_cast<cudaStream_t>(stream));       \
        });                                                                                        \
    }                                                                                              \
    int glmb_prox_step_##SFX(T* beta, const T* grad_smooth, int64_t n, double inv_L, double l1,   \
                             glmb_stream_t stream) {                                               \
        if (n < 0 || inv_L < 0 || l1 < 0) return GLMB_ERR_INVALID_VALUE;                           \
        if (n > 0 && (beta == nullptr || grad_smooth == nullptr)) return GLMB_ERR_INVALID_VALUE;   \
        return guarded([&] {                                                                       \
            return glmb::prox_step<T>(beta, grad_smooth, n, inv_L, l1,                             \
                                      reinterpret_cast<cudaStream_t>(stream));                     \
        });                                                                                        \
    }                                                                                              \
    int glmb_prox_update_##SFX(const double* partial, T* beta, const double* lipschitz,           \
                               int64_t nf, int64_t nt, int64_t ntasks, double lambda1,             \
                               double lambda2, glmb_stream_t stream) {                             \
        if (nf < 0 || nt < 0 || ntasks < 0 || lambda1 < 0 || lambda2 < 0)                          \
            return GLMB_ERR_INVALID_VALUE;                                                         \
        if (nf * nt * ntasks > 0 && (partial == nullptr || beta == nullptr || lipschitz == nullptr)) \
            return GLMB_ERR_INVALID_VALUE;                                                         \
        return guarded([&] {                                                                       \
            return glmb::prox_update<T>(partial, beta, lipschitz, nf * nt, ntasks, lambda1,        \
                                        lambda2, reinterpret_cast<cudaStream_t>(stream));          \
        });                                                                                        \
    }                                                                                              \
    int glmb_power_step_##SFX(const double* partial, T* v, double* norm, double* lipschitz,       \
                              int64_t nf, int64_t ntasks, double lambda2, glmb_stream_t stream) {  \
        if (nf < 0 || ntasks < 0 || lambda2 < 0) return GLMB_ERR_INVALID_VALUE;                    \
        if (ntasks > 0 && (partial == nullptr || v == nullptr || norm == nullptr ||                \
                           lipschitz == nullptr))                                                  \
            return GLMB_ERR_INVALID_VALUE;                                                         \
        if (ntasks > 0x7fffffff) return GLMB_ERR_TOO_LARGE;                                        \
        return guarded([&] {                                                                       \
            return glmb::power_step<T>(partial, v, norm, lipschitz, nf, ntasks, lambda2,           \
                                       reinterpret_cast<cudaStream_t>(stream));                    \
        });                                                                                        \
    }                                                                                              \
    int glmb_power_init_##SFX(T* v, int64_t nf, int64_t ntasks, uint64_t seed,                    \
                              glmb_stream_t stream) {                                              \
        if (nf < 0 || ntasks < 0) return GLMB_ERR_INVALID_VALUE;                                   \
        if (nf * ntasks > 0 && v == nullptr) return GLMB_ERR_INVALID_VALUE;                        \
        if (ntasks > 0x7fffffff) return GLMB_ERR_TOO_LARGE;                                        \
        return guarded([&] {                                                                       \
            return glmb::power_init<T>(v, nf, ntasks, seed, reinterpret_cast<cudaStream_t>(stream)); \
        });                                                                                        \
    }                                                                                              \
    size_t glmb_fit_workspace_size_##SFX(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {  \
        try {                                                                                      \
            return glmb::fit_ws_impl<T>(nf, nt, ntasks, nobs);                                     \
        } catch (...) {                                                                            \
            return 0;                                                                              \
        }                                                                                          \
    }                                                                                              \
    int glmb_fit_elastic_net_##SFX(const T* X, const T* Y, T* beta, double* lipschitz,            \
                                   int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,           \
                                   double lambda1, double lambda2, int n_power, int n_iter,        \
                                   uint64_t seed, void* workspace, size_t workspace_bytes,         \
                                   glmb_stream_t stream) {                                         \
        if (ntasks > 0x7fffffff) return GLMB_ERR_TOO_LARGE;                                        \
        return guarded([&] {                                                                       \
            return glmb::fit_impl<T>(X, Y, beta, lipschitz, nf, nt, ntasks, nobs, lambda1,         \
                                     lambda2, n_power, n_iter, seed, workspace, workspace_bytes,   \
                                     reinterpret_cast<cudaStream_t>(stream));                      \
        });                                                                                        \
    }

GLMB_DEFINE_FLOATING(f32, float)
GLMB_DEFINE_FLOATING(f64, double)

int glmb_peer_group_create(int rank, int world, int64_t max_elems, double timeout_ms, glmb_peer_group** group,
                           void* handle_out) {
    return guarded([&] { return glmb::peer_group_create(rank, world, max_elems, timeout_ms, group, handle_out); });
}
int glmb_peer_group_connect(glmb_peer_group* group, const void* handles) {
    if (handles == nullptr) return GLMB_ERR_INVALID_VALUE;
    return guarded([&] { return glmb::peer_group_connect(group, handles, nullptr); });
}
int glmb_peer_group_connect_local(glmb_peer_group* group, void* const* peer_buffers) {
    if (peer_buffers == nullptr) return GLMB_ERR_INVALID_VALUE;
    return guarded([&] { return glmb::peer_group_connect(group, nullptr, peer_buffers); });
}
void* glmb_peer_group_buffer(glmb_peer_group* group) { return glmb::peer_group_buffer(group); }
int glmb_peer_group_status(glmb_peer_group* group, int* status, int reset) {
    return guarded([&] { return glmb::peer_group_status(group, status, reset); });
}
int glmb_peer_group_destroy(glmb_peer_group* group) {
    return guarded([&] { return glmb::peer_group_destroy(group); });
}

#define GLMB_DEFINE_SHARDED_FIT(SFX, T)                                                             \
    int glmb_fit_elastic_net_sharded_##SFX(const T* X, const T* Y, T* beta, double* lipschitz,     \
                                           int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,    \
                                           double lambda1, double lambda2, int n_power, int n_iter, \
                                           uint64_t seed, glmb_peer_group* group, void* workspace,  \
                                           size_t workspace_bytes, glmb_stream_t stream) {          \
        if (group == nullptr) return GLMB_ERR_INVALID_VALUE;                                        \
        if (ntasks > 0x7fffffff) return GLMB_ERR_TOO_LARGE;                                         \
        return guarded([&] {                                                                        \
            return glmb::fit_impl<T>(X, Y, beta, lipschitz, nf, nt, ntasks, nobs, lambda1, lambda2, \
                                     n_power, n_iter, seed, workspace, workspace_bytes,             \
                                     reinterpret_cast<cudaStream_t>(stream), group);               \
        });                                                                                         \
    }

GLMB_DEFINE_SHARDED_FIT(f32, float)
GLMB_DEFINE_SHARDED_FIT(f64, double)

#define GLMB_DEFINE_PEER(SFX, T)                                                                    \
    int glmb_gradient_sharded_##SFX(const T* X, const T* M, const T* Y, T* grad_M, double* partial_out, \
                                    T* Yhat, int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,  \
                                    double lambda, double alpha, uint32_t flags, glmb_peer_group* group, \
                                    void* workspace, size_t workspace_bytes, glmb_stream_t stream) {  \
        if (group == nullptr) return GLMB_ERR_INVALID_VALUE;                                        \
        if (partial_out == nullptr && grad_M == nullptr && nf > 0 && nt > 0 && ntasks > 0)          \
            return GLMB_ERR_INVALID_VALUE;                                                          \
        return guarded([&] {                                                                        \
            return glmb::gradient_impl<T>(X, M, Y, partial_out ? nullptr : grad_M, Yhat, partial_out, nf, \
                                          nt, ntasks, nobs, lambda, alpha, flags, workspace,        \
                                          workspace_bytes, reinterpret_cast<cudaStream_t>(stream), group); \
        });                                                                                         \
    }

GLMB_DEFINE_PEER(f32, float)
GLMB_DEFINE_PEER(f64, double)

// The sharded family for the 16-bit types (uint16_t bit patterns at the ABI):
// the same partial / finalize / peer-exchange bodies on __half and bfloat16.
#define GLMB_DEFINE_SHARDED16(SFX, NT_)                                                              \
    int glmb_gradient_partial_##SFX(const uint16_t* X, const uint16_t* M, const uint16_t* Y, double* partial, \
                                    uint16_t* Yhat, int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, \
                                    uint32_t flags, void* workspace, size_t workspace_bytes,        \
                                    glmb_stream_t stream) {                                         \
        if (partial == nullptr && nf > 0 && nt > 0 && ntasks > 0) return GLMB_ERR_INVALID_VALUE;    \
        return guarded([&] {                                                                        \
            return glmb::gradient_impl<NT_>(                                                        \
                reinterpret_cast<const NT_*>(X), reinterpret_cast<const NT_*>(M),                   \
                reinterpret_cast<const NT_*>(Y), nullptr, reinterpret_cast<NT_*>(Yhat), partial, nf, nt, \
                ntasks, nobs, 0.0, 0.0, flags & ~GLMB_GRAD_REGULARIZE, workspace, workspace_bytes,  \
                reinterpret_cast<cudaStream_t>(stream));                                            \
        });                                                                                         \
    }                                                                                               \
    int glmb_gradient_finalize_##SFX(const double* partial, const uint16_t* M, uint16_t* grad_M, int64_t nf, \
                                     int64_t nt, int64_t ntasks, double lambda, double alpha,       \
                                     uint32_t flags, glmb_stream_t stream) {                        \
        if (nf < 0 || nt < 0 || ntasks < 0) return GLMB_ERR_INVALID_VALUE;                          \
        const int64_t total = nf * nt * ntasks;                                                     \
        if (total == 0) return GLMB_OK;                                                             \
        if (partial == nullptr || M == nullptr || grad_M == nullptr) return GLMB_ERR_INVALID_VALUE; \
        return guarded([&] {                                                                        \
            const int st = glmb::check_device();                                                    \
            if (st != GLMB_OK) return st;                                                           \
            return glmb::finalize_launch<NT_, double>(partial, 1, total, reinterpret_cast<const NT_*>(M), \
                                                      reinterpret_cast<NT_*>(grad_M), nullptr, lambda, alpha, \
                                                      (flags & GLMB_GRAD_REGULARIZE) != 0,           \
                                                      reinterpret_cast<cudaStream_t>(stream));      \
        });                                                                                         \
    }                                                                                               \
    int glmb_gradient_sharded_##SFX(const uint16_t* X, const uint16_t* M, const uint16_t* Y, uint16_t* grad_M, \
                                    double* partial_out, uint16_t* Yhat, int64_t nf, int64_t nt, int64_t ntasks, \
                                    int64_t nobs, double lambda, double alpha, uint32_t flags,      \
                                    glmb_peer_group* group, void* workspace, size_t workspace_bytes, \
                                    glmb_stream_t stream) {                                         \
        if (group == nullptr) return GLMB_ERR_INVALID_VALUE;                                        \
        if (partial_out == nullptr && grad_M == nullptr && nf > 0 && nt > 0 && ntasks > 0)          \
            return GLMB_ERR_INVALID_VALUE;                                                          \
        return guarded([&] {                                                                        \
            return glmb::gradient_impl<NT_>(                                                        \
                reinterpret_cast<const NT_*>(X), reinterpret_cast<const NT_*>(M),                   \
                reinterpret_cast<const NT_*>(Y), partial_out ? nullptr : reinterpret_cast<NT_*>(grad_M), \
                reinterpret_cast<NT_*>(Yhat), partial_out, nf, nt, ntasks, nobs, lambda, alpha, flags, \
                workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), group);         \
        });                                                                                         \
    }

GLMB_DEFINE_SHARDED16(f16, __half)
GLMB_DEFINE_SHARDED16(bf16, __nv_bfloat16)

}  // extern "C"
