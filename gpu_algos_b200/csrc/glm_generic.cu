// glm_generic.cu -- element-type-generic GLM kernels and the shared
// fixed-order reduction (see glm_generic.cuh).
#include <algorithm>

#include "glm_generic.cuh"

namespace glmb {

namespace {

constexpr int kGenTX = 32;  // features per block (one per lane)
constexpr int kGenTY = 8;   // observation lanes per block
constexpr int kGenTT = 8;   // targets per register tile

// One thread per (obs, task, target): yhat = <X row, M row>, E = yhat - y.
// logistic (float/double): yhat = sigmoid(<X row, M row>), E = (yhat - y) / 2
// (the finalize's factor 2 then gives the logistic log-likelihood gradient).
template <typename T>
__global__ void __launch_bounds__(256)
    glm_residual_kernel(const T* __restrict__ X, const T* __restrict__ M, const T* __restrict__ Y,
                        T* __restrict__ Yhat, typename Arith<T>::Dot* __restrict__ E, int64_t nf,
                        int64_t nt, int64_t ntasks, int64_t nobs, int logistic) {
    using D = typename Arith<T>::Dot;
    const int64_t n = nobs * ntasks * nt;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t t = i % nt;
        const int64_t row = i / nt;
        const int64_t task = row % ntasks;
        const T* x = X + row * nf;
        const T* m = M + (task * nt + t) * nf;
        if constexpr (std::is_floating_point_v<D>) {
            // one dot product per output, as accurate as the output type can
            // hold: float products are exact in double; double uses the
            // compensated dot product (error-free product and sum of every
            // term, Ogita, Rump & Oishi 2005), so the result is as if carried
            // in twice the working precision
            double d;
            if constexpr (std::is_same_v<D, double>) {
                double s = 0.0, c = 0.0;
                for (int64_t f = 0; f < nf; ++f) {
                    const double a = to_arith<double>(m[f]), b = to_arith<double>(x[f]);
                    const double p = a * b;
                    const double ep = fma(a, b, -p);
                    const double u = s + p;
                    const double z = u - s;
                    const double es = (s - (u - z)) + (p - z);
                    s = u;
                    c += ep + es;
                }
                d = s + c;
            } else {
                d = 0.0;
                for (int64_t f = 0; f < nf; ++f) d = fma(to_arith<double>(m[f]), to_arith<double>(x[f]), d);
            }
            if (logistic) d = sigmoid(d);
            if (Yhat != nullptr) Yhat[i] = from_arith<T>(D(d));
            if (E != nullptr) {
                const double e = d - (Y != nullptr ? to_arith<double>(Y[i]) : 0.0);
                E[i] = D(logistic ? 0.5 * e : e);
            }
        } else {
            D d = D(0);
            for (int64_t f = 0; f < nf; ++f) d += to_arith<D>(m[f]) * to_arith<D>(x[f]);
            if (Yhat != nullptr) Yhat[i] = from_arith<T>(d);
            if (E != nullptr) E[i] = d - (Y != nullptr ? to_arith<D>(Y[i]) : D(0));
        }
    }
}

// Block (32 features x 8 obs lanes) over one (feature block, task, obs split):
// part[(task*K + t*nf + f) * nsplit + split] = sum_obs E[obs,task,t] * X[obs,task,f].
template <typename T>
__global__ void __launch_bounds__(kGenTX* kGenTY)
    glm_xtr_kernel(const T* __restrict__ X, const typename Arith<T>::Dot* __restrict__ E,
                   typename Arith<T>::Acc* __restrict__ part, int64_t nf, int64_t nt,
                   int64_t ntasks, int64_t nobs, int64_t obs_per_split, int64_t nfblk) {
    using A = typename Arith<T>::Acc;
    __shared__ A red[kGenTY][kGenTT][kGenTX];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int64_t fblk = blockIdx.x % nfblk;
    const int64_t task = blockIdx.x / nfblk;
    const int64_t f = fblk * kGenTX + tx;
    const int64_t split = blockIdx.y;
    const int64_t nsplit = gridDim.y;
    const int64_t o0 = split * obs_per_split;
    const int64_t o1 = min(nobs, o0 + obs_per_split);
    const int64_t K = nt * nf;
    for (int64_t t0 = 0; t0 < nt; t0 += kGenTT) {
        A acc[kGenTT];
#pragma unroll
        for (int j = 0; j < kGenTT; ++j) acc[j] = A(0);
        for (int64_t obs = o0 + ty; obs < o1; obs += kGenTY) {
            const int64_t row = obs * ntasks + task;
            const A x = f < nf ? to_arith<A>(X[row * nf + f]) : A(0);
#pragma unroll
            for (int j = 0; j < kGenTT; ++j)
                if (t0 + j < nt) acc[j] += static_cast<A>(E[row * nt + t0 + j]) * x;
        }
#pragma unroll
        for (int j = 0; j < kGenTT; ++j) red[ty][j][tx] = acc[j];
        __syncthreads();
        if (ty == 0) {
#pragma unroll
            for (int j = 0; j < kGenTT; ++j) {
                A s = red[0][j][tx];
#pragma unroll
                for (int y = 1; y < kGenTY; ++y) s += red[y][j][tx];
                if (f < nf && t0 + j < nt) part[(task * K + (t0 + j) * nf + f) * nsplit + split] = s;
            }
        }
        __syncthreads();
    }
}

template <typename T, typename P>
__global__ void __launch_bounds__(256)
    glm_finalize_kernel(const P* __restrict__ part, int64_t nparts, int64_t total,
                        const T* __restrict__ M, T* __restrict__ grad, double* __restrict__ partial_out,
                        double lambda, double alpha, int reg) {
    pdl_wait_for_producer();  // the partials are the previous kernel's output
    const int lane = threadIdx.x & (kWarp - 1);
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t e = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; e < total; e += nwarps) {
        P s = P(0);
        // unrolled: eight independent loads in flight, the additions in the same order
#pragma unroll 8
        for (int64_t c = lane; c < nparts; c += kWarp) s += part[e * nparts + c];
#pragma unroll
        for (int off = kWarp / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) {
            if (partial_out != nullptr) {
                partial_out[e] = static_cast<double>(s);
            } else {
                grad[e] = finalize_value<T>(s, M[e], lambda, alpha, reg != 0);
            }
        }
    }
}

struct GenericPlan {
    int64_t nfblk = 0, nsplit = 0, obs_per_split = 0;
    size_t e_bytes = 0, part_bytes = 0;
};

template <typename T>
GenericPlan generic_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {
    using D = typename Arith<T>::Dot;
    using A = typename Arith<T>::Acc;
    GenericPlan p;
    p.nfblk = (nf + kGenTX - 1) / kGenTX;
    const int64_t blocks_xy = std::max<int64_t>(1, p.nfblk * ntasks);
    const int64_t want = (4 * int64_t(sm_count()) + blocks_xy - 1) / blocks_xy;
    const int64_t most = std::max<int64_t>(1, (nobs + 63) / 64);
    p.nsplit = nobs > 0 ? std::min<int64_t>({std::max<int64_t>(1, want), most, 65535}) : 0;
    p.obs_per_split = p.nsplit > 0 ? (nobs + p.nsplit - 1) / p.nsplit : 0;
    if (p.nsplit > 0) p.nsplit = (nobs + p.obs_per_split - 1) / p.obs_per_split;
    p.e_bytes = round_up(size_t(nobs) * ntasks * nt * sizeof(D), 256);
    p.part_bytes = round_up(size_t(ntasks) * nt * nf * std::max<int64_t>(1, p.nsplit) * sizeof(A), 256);
    return p;
}

inline unsigned grid_for(int64_t n, int threads) {
    const int64_t cap = int64_t(sm_count()) * 16;
    return unsigned(std::max<int64_t>(1, std::min<int64_t>(cap, (n + threads - 1) / threads)));
}

}  // namespace

template <typename T>
size_t generic_workspace_bytes(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {
    const GenericPlan p = generic_plan<T>(nf, nt, ntasks, nobs);
    return p.e_bytes + p.part_bytes;
}

template <typename T>
int generic_predict(const T* X, const T* M, T* Yhat, int64_t nf, int64_t nt, int64_t ntasks,
                    int64_t nobs, cudaStream_t stream) {
    const int64_t n = nobs * ntasks * nt;
    if (n == 0) return GLMB_OK;
    glm_residual_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(X, M, nullptr, Yhat, nullptr, nf,
                                                                  nt, ntasks, nobs, 0);
    count_launch();
    return launch_status();
}

template <typename T, typename P>
int finalize_launch(const P* part, int64_t nparts, int64_t total, const T* M, T* grad,
                    double* partial_out, double lambda, double alpha, bool reg,
                    cudaStream_t stream) {
    if (total == 0) return GLMB_OK;
    const int64_t warps_per_block = 256 / kWarp;
    const unsigned blocks = unsigned(std::max<int64_t>(
        1, std::min<int64_t>(int64_t(sm_count()) * 8, (total + warps_per_block - 1) / warps_per_block)));
    const cudaError_t e = pdl_launch(glm_finalize_kernel<T, P>, dim3(blocks), dim3(256), 0, stream, part, nparts,
                                     total, M, grad, partial_out, lambda, alpha, reg ? 1 : 0);
    count_launch();
    if (e != cudaSuccess) return int(e);
    return launch_status();
}

template <typename T>
int generic_gradient(const T* X, const T* M, const T* Y, T* grad, T* Yhat, double* partial_out,
                     int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, double lambda,
                     double alpha, bool reg, void* ws, size_t ws_bytes, cudaStream_t stream,
                     PartsFinisher fin, void* fin_ctx, bool logistic) {
    using D = typename Arith<T>::Dot;
    using A = typename Arith<T>::Acc;
    const GenericPlan p = generic_plan<T>(nf, nt, ntasks, nobs);
    Scratch sc(ws, ws_bytes, p.e_bytes + p.part_bytes, stream);
    if (sc.status() != GLMB_OK) return sc.status();
    D* E = sc.as<D>();
    A* part = reinterpret_cast<A*>(sc.as<char>() + p.e_bytes);
    int st = GLMB_OK;
    const int64_t n = nobs * ntasks * nt;
    if (n > 0) {
        glm_residual_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(X, M, Y, Yhat, E, nf, nt,
                                                                      ntasks, nobs, logistic ? 1 : 0);
        count_launch();
        if ((st = launch_status()) != GLMB_OK) return st;
    }
    if (p.nsplit > 0) {
        const dim3 grid(unsigned(p.nfblk * ntasks), unsigned(p.nsplit));
        glm_xtr_kernel<T><<<grid, dim3(kGenTX, kGenTY), 0, stream>>>(X, E, part, nf, nt, ntasks, nobs,
                                                                     p.obs_per_split, p.nfblk);
        count_launch();
        if ((st = launch_status()) != GLMB_OK) return st;
    }
    if (fin != nullptr) return fin(fin_ctx, part, p.nsplit);
    return finalize_launch<T, A>(part, p.nsplit, ntasks * nt * nf, M, grad, partial_out, lambda,
                                 alpha, reg, stream);
}

#define GLMB_INSTANTIATE_GENERIC(T)                                                                \
    template size_t generic_workspace_bytes<T>(int64_t, int64_t, int64_t, int64_t);                \
    template int generic_predict<T>(const T*, const T*, T*, int64_t, int64_t, int64_t, int64_t,    \
                                    cudaStream_t);                                                 \
    template int generic_gradient<T>(const T*, const T*, const T*, T*, T*, double*, int64_t,       \
                                     int64_t, int64_t, int64_t, double, double, bool, void*,       \
                                     size_t, cudaStream_t, PartsFinisher, void*, bool);

GLMB_INSTANTIATE_GENERIC(__half)
GLMB_INSTANTIATE_GENERIC(__nv_bfloat16)
GLMB_INSTANTIATE_GENERIC(float)
GLMB_INSTANTIATE_GENERIC(double)
GLMB_INSTANTIATE_GENERIC(int8_t)
GLMB_INSTANTIATE_GENERIC(int16_t)
GLMB_INSTANTIATE_GENERIC(int32_t)
GLMB_INSTANTIATE_GENERIC(int64_t)
GLMB_INSTANTIATE_GENERIC(uint8_t)
GLMB_INSTANTIATE_GENERIC(uint16_t)
GLMB_INSTANTIATE_GENERIC(uint32_t)
GLMB_INSTANTIATE_GENERIC(uint64_t)

template int finalize_launch<__half, double>(const double*, int64_t, int64_t, const __half*, __half*,
                                             double*, double, double, bool, cudaStream_t);
template int finalize_launch<__nv_bfloat16, double>(const double*, int64_t, int64_t, const __nv_bfloat16*,
                                                    __nv_bfloat16*, double*, double, double, bool, cudaStream_t);
template int finalize_launch<float, double>(const double*, int64_t, int64_t, const float*, float*,
                                            double*, double, double, bool, cudaStream_t);
template int finalize_launch<double, double>(const double*, int64_t, int64_t, const double*,
                                             double*, double*, double, double, bool, cudaStream_t);

}  // namespace glmb
