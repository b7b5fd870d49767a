// glm_mg.cu -- single-process multi-GPU context for C and C++ hosts.
//
// The reference is single-GPU: a host thread calls run_device_kernel on one
// stream (include/cuda/kernels/glm/glm_gradient_xyyhat.cuh:642).  A C++ host
// that owns several GPUs uses this context instead: observations are split
// into one contiguous block per device (the caller places block i on device
// i), each device computes its block's partial sum
//     P_i = sum_{obs in block i} (Yhat - Y) X      (double)
// and the partials are summed across the devices by one of two exchanges:
//   GLMB_MG_PEER  the library's exchange kernel over NVLink peer memory
//                 (glm_peer.cu; CUDA peer access between the devices);
//   GLMB_MG_NCCL  ncclAllReduce on one communicator per device
//                 (ncclCommInitAll); NCCL is loaded when the context is
//                 created (dlopen of libnccl.so.2), so the library has no
//                 link-time dependency on it.
// Every device then applies the same finalize (2*sum + elastic-net term), so
// all devices hold bit-identical gradients.  The sharded elastic-net fit runs
// the same exchange for every power iteration and ISTA step, with the
// launches of each iteration issued device by device: an exchange kernel
// waits for its peers' partials, and every device's part of an iteration is
// enqueued before the next iteration's.
//
// One host thread drives all devices; every call is asynchronous on the
// context's streams (one per device) and leaves the caller's current device
// as it found it.  glmb_mg_synchronize waits for them and reports an
// exchange whose wait ran out.  A context is not re-entrant: calls on one
// context must not overlap from several host threads.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <new>
#include <vector>

#include "glm_common.cuh"
#include "glm_fit.cuh"
#include "glm_generic.cuh"
#include "glm_peer.cuh"

namespace glmb {
template <typename T>
int sharded_gradient(const T* X, const T* M, const T* Y, T* grad, double* partial_out, int64_t nf, int64_t nt,
                     int64_t ntasks, int64_t nobs, double lambda, double alpha, uint32_t flags,
                     cudaStream_t stream, glmb_peer_group* group);
int device_check();
}  // namespace glmb

namespace {

// The NCCL entry points the context uses, resolved from libnccl.so.2.
struct NcclApi {
    void* lib = nullptr;
    ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;

    bool load() {
        lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (lib == nullptr) return false;
        comm_init_all = reinterpret_cast<decltype(comm_init_all)>(dlsym(lib, "ncclCommInitAll"));
        all_reduce = reinterpret_cast<decltype(all_reduce)>(dlsym(lib, "ncclAllReduce"));
        group_start = reinterpret_cast<decltype(group_start)>(dlsym(lib, "ncclGroupStart"));
        group_end = reinterpret_cast<decltype(group_end)>(dlsym(lib, "ncclGroupEnd"));
        comm_destroy = reinterpret_cast<decltype(comm_destroy)>(dlsym(lib, "ncclCommDestroy"));
        return comm_init_all && all_reduce && group_start && group_end && comm_destroy;
    }
};

// Restores the caller's current device when a call returns.
struct DeviceGuard {
    int saved = -1;
    DeviceGuard() {
        if (cudaGetDevice(&saved) != cudaSuccess) saved = -1;
    }
    ~DeviceGuard() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};

}  // namespace

struct glmb_mg {
    int n = 0;
    uint32_t mode = GLMB_MG_PEER;
    int64_t max_elems = 0;
    int dev[GLMB_MG_MAX_DEVICES] = {};
    cudaStream_t stream[GLMB_MG_MAX_DEVICES] = {};
    glmb_peer_group* group[GLMB_MG_MAX_DEVICES] = {};
    ncclComm_t comm[GLMB_MG_MAX_DEVICES] = {};
    NcclApi nccl;
};

namespace glmb {
namespace {

int mg_destroy(glmb_mg* mg) {
    if (mg == nullptr) return GLMB_OK;
    DeviceGuard keep;
    int st = GLMB_OK;
    for (int i = 0; i < mg->n; ++i) {
        if (cudaSetDevice(mg->dev[i]) != cudaSuccess) continue;
        if (mg->stream[i] != nullptr) cudaStreamSynchronize(mg->stream[i]);
        if (mg->comm[i] != nullptr && mg->nccl.comm_destroy != nullptr) mg->nccl.comm_destroy(mg->comm[i]);
        if (mg->group[i] != nullptr) {
            const int s = peer_group_destroy(mg->group[i]);
            if (s != GLMB_OK && st == GLMB_OK) st = s;
        }
        if (mg->stream[i] != nullptr) cudaStreamDestroy(mg->stream[i]);
    }
    if (mg->nccl.lib != nullptr) dlclose(mg->nccl.lib);
    delete mg;
    return st;
}

int mg_create(int ndev, const int* devices, int64_t max_elems, double timeout_ms, uint32_t mode, glmb_mg** out) {
    if (out == nullptr) return GLMB_ERR_INVALID_VALUE;
    *out = nullptr;
    if (ndev < 1 || ndev > GLMB_MG_MAX_DEVICES || devices == nullptr || max_elems < 1 || timeout_ms <= 0 ||
        (mode != GLMB_MG_PEER && mode != GLMB_MG_NCCL))
        return GLMB_ERR_INVALID_VALUE;
    for (int i = 0; i < ndev; ++i)
        for (int j = 0; j < i; ++j)
            if (devices[i] == devices[j]) return GLMB_ERR_INVALID_VALUE;  // one block per device
    DeviceGuard keep;
    auto* mg = new (std::nothrow) glmb_mg();
    if (mg == nullptr) return GLMB_ERR_INVALID_VALUE;
    mg->mode = mode;
    mg->max_elems = max_elems;
    auto fail = [&](int st) {
        mg_destroy(mg);
        return st;
    };
    for (int i = 0; i < ndev; ++i) {
        mg->dev[i] = devices[i];
        cudaError_t e = cudaSetDevice(devices[i]);
        if (e != cudaSuccess) return fail(int(e));
        const int chk = device_check();
        if (chk != GLMB_OK) return fail(chk);
        e = cudaStreamCreateWithFlags(&mg->stream[i], cudaStreamNonBlocking);
        mg->n = i + 1;
        if (e != cudaSuccess) return fail(int(e));
    }
    if (mode == GLMB_MG_PEER) {
        // every device reaches every other device's exchange buffer directly
        for (int i = 0; i < ndev; ++i) {
            cudaSetDevice(devices[i]);
            for (int j = 0; j < ndev; ++j) {
                if (j == i) continue;
                int can = 0;
                cudaError_t e = cudaDeviceCanAccessPeer(&can, devices[i], devices[j]);
                if (e != cudaSuccess) return fail(int(e));
                if (!can) return fail(GLMB_ERR_UNSUPPORTED);
                e = cudaDeviceEnablePeerAccess(devices[j], 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) {
                    cudaGetLastError();
                } else if (e != cudaSuccess) {
                    return fail(int(e));
                }
            }
        }
        void* bufs[GLMB_MG_MAX_DEVICES] = {};
        for (int i = 0; i < ndev; ++i) {
            cudaSetDevice(devices[i]);
            const int st = peer_group_create(i, ndev, max_elems, timeout_ms, &mg->group[i], nullptr);
            if (st != GLMB_OK) return fail(st);
            bufs[i] = peer_group_buffer(mg->group[i]);
        }
        for (int i = 0; i < ndev; ++i) {
            cudaSetDevice(devices[i]);
            const int st = peer_group_connect(mg->group[i], nullptr, bufs);
            if (st != GLMB_OK) return fail(st);
        }
    } else {
        if (!mg->nccl.load()) return fail(GLMB_ERR_UNSUPPORTED);
        if (mg->nccl.comm_init_all(mg->comm, ndev, devices) != ncclSuccess) {
            for (int i = 0; i < ndev; ++i) mg->comm[i] = nullptr;
            return fail(GLMB_ERR_COLLECTIVE);
        }
    }
    *out = mg;
    return GLMB_OK;
}

int mg_synchronize(glmb_mg* mg) {
    if (mg == nullptr) return GLMB_ERR_INVALID_VALUE;
    DeviceGuard keep;
    int st = GLMB_OK;
    for (int i = 0; i < mg->n; ++i) {
        cudaError_t e = cudaSetDevice(mg->dev[i]);
        if (e == cudaSuccess) e = cudaStreamSynchronize(mg->stream[i]);
        if (e != cudaSuccess && st == GLMB_OK) st = int(e);
        if (mg->group[i] != nullptr) {
            int s = 0;
            const int r = peer_group_status(mg->group[i], &s, 1);
            if (r != GLMB_OK && st == GLMB_OK) st = r;
            if (s != 0 && st == GLMB_OK) st = GLMB_ERR_PEER_TIMEOUT;
        }
    }
    return st;
}

// Per-device scratch of one call, released in stream order when the call returns.
struct DeviceScratch {
    std::vector<void*> ptr;
    glmb_mg* mg;
    explicit DeviceScratch(glmb_mg* m) : ptr(size_t(m->n), nullptr), mg(m) {}
    int alloc(int i, size_t bytes) {
        cudaSetDevice(mg->dev[i]);
        return int(cudaMallocAsync(&ptr[size_t(i)], bytes, mg->stream[i]));
    }
    ~DeviceScratch() {
        for (int i = 0; i < mg->n; ++i)
            if (ptr[size_t(i)] != nullptr) {
                cudaSetDevice(mg->dev[i]);
                cudaFreeAsync(ptr[size_t(i)], mg->stream[i]);
            }
    }
};

int mg_check_shards(glmb_mg* mg, const int64_t* nobs, int64_t nf, int64_t nt, int64_t ntasks) {
    if (mg == nullptr || nobs == nullptr || nf < 0 || nt < 0 || ntasks < 0) return GLMB_ERR_INVALID_VALUE;
    for (int i = 0; i < mg->n; ++i)
        if (nobs[i] < 0) return GLMB_ERR_INVALID_VALUE;
    if (nf * nt * ntasks > mg->max_elems) return GLMB_ERR_TOO_LARGE;
    return GLMB_OK;
}

// The summed partial of every device's block, on every device: the peer
// exchange writes it directly; NCCL sums the local partials in place.
template <typename T>
int mg_partial_all(glmb_mg* mg, const T* const* X, const T* const* M, const T* const* Y, double* const* part,
                   const int64_t* nobs, int64_t nf, int64_t nt, int64_t ntasks, uint32_t flags) {
    const int64_t total = nf * nt * ntasks;
    for (int i = 0; i < mg->n; ++i) {
        cudaError_t e = cudaSetDevice(mg->dev[i]);
        if (e != cudaSuccess) return int(e);
        const int st = sharded_gradient<T>(X[i], M[i], Y ? Y[i] : nullptr, nullptr, part[i], nf, nt, ntasks, nobs[i],
                                           0.0, 0.0, flags & ~uint32_t(GLMB_GRAD_REGULARIZE), mg->stream[i],
                                           mg->mode == GLMB_MG_PEER ? mg->group[i] : nullptr);
        if (st != GLMB_OK) return st;
    }
    if (mg->mode == GLMB_MG_NCCL) {
        if (mg->nccl.group_start() != ncclSuccess) return GLMB_ERR_COLLECTIVE;
        int st = GLMB_OK;
        for (int i = 0; i < mg->n; ++i)
            if (mg->nccl.all_reduce(part[i], part[i], size_t(total), ncclDouble, ncclSum, mg->comm[i],
                                    mg->stream[i]) != ncclSuccess)
                st = GLMB_ERR_COLLECTIVE;
        if (mg->nccl.group_end() != ncclSuccess) st = GLMB_ERR_COLLECTIVE;
        if (st != GLMB_OK) return st;
    }
    return GLMB_OK;
}

template <typename T>
int mg_gradient(glmb_mg* mg, const T* const* X, const T* const* M, const T* const* Y, T* const* grad,
                const int64_t* nobs, int64_t nf, int64_t nt, int64_t ntasks, double lambda, double alpha,
                uint32_t flags) {
    int st = mg_check_shards(mg, nobs, nf, nt, ntasks);
    if (st != GLMB_OK) return st;
    if (flags & ~uint32_t(GLMB_GRAD_REGULARIZE | GLMB_GRAD_Y_ZERO | GLMB_GRAD_LOGISTIC)) return GLMB_ERR_INVALID_VALUE;
    if (X == nullptr || M == nullptr || grad == nullptr || (Y == nullptr && !(flags & GLMB_GRAD_Y_ZERO)))
        return GLMB_ERR_INVALID_VALUE;
    const int64_t total = nf * nt * ntasks;
    if (total == 0) return GLMB_OK;
    DeviceGuard keep;
    const bool reg = (flags & GLMB_GRAD_REGULARIZE) != 0;
    if (mg->mode == GLMB_MG_PEER) {
        // partial + exchange + finalize in the exchange kernel, device by device
        for (int i = 0; i < mg->n; ++i) {
            cudaError_t e = cudaSetDevice(mg->dev[i]);
            if (e != cudaSuccess) return int(e);
            st = sharded_gradient<T>(X[i], M[i], (flags & GLMB_GRAD_Y_ZERO) ? nullptr : Y[i], grad[i], nullptr, nf,
                                     nt, ntasks, nobs[i], lambda, alpha, flags, mg->stream[i], mg->group[i]);
            if (st != GLMB_OK) return st;
        }
        return GLMB_OK;
    }
    DeviceScratch part(mg);
    std::vector<double*> P(size_t(mg->n));
    for (int i = 0; i < mg->n; ++i) {
        if ((st = part.alloc(i, size_t(total) * sizeof(double))) != GLMB_OK) return st;
        P[size_t(i)] = static_cast<double*>(part.ptr[size_t(i)]);
    }
    st = mg_partial_all<T>(mg, X, M, (flags & GLMB_GRAD_Y_ZERO) ? nullptr : Y, P.data(), nobs, nf, nt, ntasks, flags);
    if (st != GLMB_OK) return st;
    for (int i = 0; i < mg->n; ++i) {
        cudaSetDevice(mg->dev[i]);
        st = finalize_launch<T, double>(P[size_t(i)], 1, total, M[i], grad[i], nullptr, lambda, alpha, reg,
                                        mg->stream[i]);
        if (st != GLMB_OK) return st;
    }
    return GLMB_OK;
}

template <typename T>
int mg_fit(glmb_mg* mg, const T* const* X, const T* const* Y, T* const* beta, double* const* lipschitz,
           const int64_t* nobs, int64_t nf, int64_t nt, int64_t ntasks, double lambda1, double lambda2, int n_power,
           int n_iter, uint64_t seed) {
    int st = mg_check_shards(mg, nobs, nf, std::max<int64_t>(nt, 1), ntasks);
    if (st != GLMB_OK) return st;
    if (n_power < 0 || n_iter < 0 || lambda1 < 0 || lambda2 < 0 || (n_iter > 0 && n_power < 1))
        return GLMB_ERR_INVALID_VALUE;
    if (nf == 0 || nt == 0 || ntasks == 0) return GLMB_OK;
    if (X == nullptr || Y == nullptr || beta == nullptr || lipschitz == nullptr) return GLMB_ERR_INVALID_VALUE;
    DeviceGuard keep;
    const int64_t K = nt * nf;
    // per device: summed partial (ntasks*nt*nf doubles), power vector v (ntasks*nf), its norm (ntasks)
    const size_t part_bytes = round_up(size_t(ntasks * K) * sizeof(double), 256);
    const size_t v_bytes = round_up(size_t(ntasks * nf) * sizeof(T), 256);
    const size_t norm_bytes = round_up(size_t(ntasks) * sizeof(double), 256);
    DeviceScratch sc(mg);
    std::vector<double*> P(size_t(mg->n)), norm(size_t(mg->n));
    std::vector<T*> v(size_t(mg->n));
    std::vector<const T*> vc(size_t(mg->n)), bc(size_t(mg->n));
    for (int i = 0; i < mg->n; ++i) {
        if ((st = sc.alloc(i, part_bytes + v_bytes + norm_bytes)) != GLMB_OK) return st;
        char* base = static_cast<char*>(sc.ptr[size_t(i)]);
        P[size_t(i)] = reinterpret_cast<double*>(base);
        v[size_t(i)] = reinterpret_cast<T*>(base + part_bytes);
        norm[size_t(i)] = reinterpret_cast<double*>(base + part_bytes + v_bytes);
        vc[size_t(i)] = v[size_t(i)];
        bc[size_t(i)] = beta[i];
        if ((st = power_init<T>(v[size_t(i)], nf, ntasks, seed, mg->stream[i])) != GLMB_OK) return st;
    }
    for (int it = 0; it < n_power; ++it) {
        st = mg_partial_all<T>(mg, X, vc.data(), nullptr, P.data(), nobs, nf, 1, ntasks, GLMB_GRAD_Y_ZERO);
        if (st != GLMB_OK) return st;
        for (int i = 0; i < mg->n; ++i) {
            cudaSetDevice(mg->dev[i]);
            st = power_step<T>(P[size_t(i)], v[size_t(i)], norm[size_t(i)], lipschitz[i], nf, ntasks, lambda2,
                               mg->stream[i]);
            if (st != GLMB_OK) return st;
        }
    }
    for (int i = 0; i < mg->n; ++i) {
        cudaSetDevice(mg->dev[i]);
        const cudaError_t e = cudaMemsetAsync(beta[i], 0, size_t(K * ntasks) * sizeof(T), mg->stream[i]);
        if (e != cudaSuccess) return int(e);
    }
    for (int it = 0; it < n_iter; ++it) {
        st = mg_partial_all<T>(mg, X, bc.data(), Y, P.data(), nobs, nf, nt, ntasks, 0u);
        if (st != GLMB_OK) return st;
        for (int i = 0; i < mg->n; ++i) {
            cudaSetDevice(mg->dev[i]);
            st = prox_update<T>(P[size_t(i)], beta[i], lipschitz[i], K, ntasks, lambda1, lambda2, mg->stream[i]);
            if (st != GLMB_OK) return st;
        }
    }
    return GLMB_OK;
}

template <typename F>
int mg_guarded(F&& f) {
    try {
        return f();
    } catch (...) {
        return GLMB_ERR_INVALID_VALUE;
    }
}

}  // namespace
}  // namespace glmb

extern "C" {

int glmb_mg_create(int ndev, const int* devices, int64_t max_elems, double timeout_ms, uint32_t mode,
                   glmb_mg** mg) {
    return glmb::mg_guarded([&] { return glmb::mg_create(ndev, devices, max_elems, timeout_ms, mode, mg); });
}
int glmb_mg_destroy(glmb_mg* mg) {
    return glmb::mg_guarded([&] { return glmb::mg_destroy(mg); });
}
int glmb_mg_size(glmb_mg* mg) { return mg == nullptr ? 0 : mg->n; }
int glmb_mg_stream(glmb_mg* mg, int i, glmb_stream_t* stream) {
    if (mg == nullptr || stream == nullptr || i < 0 || i >= mg->n) return GLMB_ERR_INVALID_VALUE;
    *stream = reinterpret_cast<glmb_stream_t>(mg->stream[i]);
    return GLMB_OK;
}
int glmb_mg_synchronize(glmb_mg* mg) {
    return glmb::mg_guarded([&] { return glmb::mg_synchronize(mg); });
}

#define GLMB_DEFINE_MG(SFX, T)                                                                          \
    int glmb_mg_gradient_##SFX(glmb_mg* mg, const T* const* X, const T* const* M, const T* const* Y,   \
                               T* const* grad_M, const int64_t* nobs, int64_t nf, int64_t nt,          \
                               int64_t ntasks, double lambda, double alpha, uint32_t flags) {          \
        return glmb::mg_guarded([&] {                                                                   \
            return glmb::mg_gradient<T>(mg, X, M, Y, grad_M, nobs, nf, nt, ntasks, lambda, alpha, flags); \
        });                                                                                             \
    }                                                                                                   \
    int glmb_mg_fit_elastic_net_##SFX(glmb_mg* mg, const T* const* X, const T* const* Y, T* const* beta, \
                                      double* const* lipschitz, const int64_t* nobs, int64_t nf,        \
                                      int64_t nt, int64_t ntasks, double lambda1, double lambda2,       \
                                      int n_power, int n_iter, uint64_t seed) {                         \
        return glmb::mg_guarded([&] {                                                                   \
            return glmb::mg_fit<T>(mg, X, Y, beta, lipschitz, nobs, nf, nt, ntasks, lambda1, lambda2,   \
                                   n_power, n_iter, seed);                                              \
        });                                                                                             \
    }

GLMB_DEFINE_MG(f32, float)
GLMB_DEFINE_MG(f64, double)

}  // extern "C"
