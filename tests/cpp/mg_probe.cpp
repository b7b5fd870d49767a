// mg_probe.cpp -- a C++ host driving two or more GPUs through the library's
// multi-GPU context (include/glm_b200.h: glmb_mg_*), the way a host program
// in the reference's style (C++, one thread, no torch) would.
//
// For the peer exchange and for NCCL it checks, against the one-GPU entry
// points on device 0 over the whole data:
//   - the sharded gradient (float and double), bit-identical on every device;
//   - the sharded elastic-net fit (beta and L), bit-identical on every device.
// Prints one "PASS <what>" line per check and "ALL PASS" at the end; exits
// non-zero on the first failure.  Usage: mg_probe <ndev> [peer|nccl|both]
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "glm_b200.h"

namespace {

#define CHECK_CUDA(x)                                                                            \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            std::printf("FAIL cuda %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__);  \
            std::exit(2);                                                                        \
        }                                                                                        \
    } while (0)
#define CHECK_GLMB(x)                                                                            \
    do {                                                                                         \
        int s_ = (x);                                                                            \
        if (s_ != 0) {                                                                           \
            std::printf("FAIL glmb %d (%s) at %s:%d\n", s_, glmb_status_string(s_), __FILE__,   \
                        __LINE__);                                                               \
            std::exit(3);                                                                        \
        }                                                                                        \
    } while (0)

template <typename T>
T* to_device(int dev, const T* host, size_t n) {
    CHECK_CUDA(cudaSetDevice(dev));
    T* d = nullptr;
    CHECK_CUDA(cudaMalloc(&d, std::max<size_t>(n, 1) * sizeof(T)));
    if (n) CHECK_CUDA(cudaMemcpy(d, host, n * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

template <typename T>
std::vector<T> to_host(int dev, const T* d, size_t n) {
    CHECK_CUDA(cudaSetDevice(dev));
    std::vector<T> h(n);
    CHECK_CUDA(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost));
    return h;
}

// max |a-b| / max(|b|, floor*max|b|)
double rel_err(const std::vector<double>& a, const std::vector<double>& b, double floor) {
    double mx = 0.0, worst = 0.0;
    for (double v : b) mx = std::max(mx, std::fabs(v));
    for (size_t i = 0; i < a.size(); ++i) {
        const double den = std::max(std::fabs(b[i]), floor * mx);
        worst = std::max(worst, den > 0 ? std::fabs(a[i] - b[i]) / den : std::fabs(a[i] - b[i]));
    }
    return worst;
}

template <typename T>
std::vector<double> widen(const std::vector<T>& v) {
    return std::vector<double>(v.begin(), v.end());
}

struct Problem {
    int64_t nobs, ntasks, nf, nt;
};

template <typename T>
struct Api;
template <>
struct Api<float> {
    static constexpr const char* name = "f32";
    static constexpr double tol = 1e-4;
    static auto gradient() { return &glmb_gradient_f32; }
    static auto mg_gradient() { return &glmb_mg_gradient_f32; }
    static auto fit() { return &glmb_fit_elastic_net_f32; }
    static auto mg_fit() { return &glmb_mg_fit_elastic_net_f32; }
};
template <>
struct Api<double> {
    static constexpr const char* name = "f64";
    static constexpr double tol = 1e-11;
    static auto gradient() { return &glmb_gradient_f64; }
    static auto mg_gradient() { return &glmb_mg_gradient_f64; }
    static auto fit() { return &glmb_fit_elastic_net_f64; }
    static auto mg_fit() { return &glmb_mg_fit_elastic_net_f64; }
};

template <typename T>
bool run(glmb_mg* mg, int ndev, const char* mode, const Problem& pb, uint64_t seed) {
    const int64_t nobs = pb.nobs, ntasks = pb.ntasks, nf = pb.nf, nt = pb.nt;
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<double> U(-1.0, 1.0);
    std::normal_distribution<double> N(0.0, 1.0);
    std::vector<T> X(size_t(nobs * ntasks * nf)), Y(size_t(nobs * ntasks * nt)), M(size_t(ntasks * nt * nf));
    std::vector<double> bt(size_t(ntasks * nt * nf));
    for (auto& x : X) x = T(U(rng));
    for (auto& b : bt) b = N(rng);
    for (auto& m : M) m = T(N(rng));
    for (int64_t o = 0; o < nobs; ++o)
        for (int64_t k = 0; k < ntasks; ++k)
            for (int64_t t = 0; t < nt; ++t) {
                double s = 0.0;
                for (int64_t f = 0; f < nf; ++f)
                    s += double(X[size_t((o * ntasks + k) * nf + f)]) * bt[size_t((k * nt + t) * nf + f)];
                Y[size_t((o * ntasks + k) * nt + t)] = T(s + 0.1 * N(rng));
            }
    const size_t K = size_t(ntasks * nt * nf);
    const double lam = 0.2, alpha = 0.3;

    // one GPU, the whole data
    T *dX = to_device(0, X.data(), X.size()), *dY = to_device(0, Y.data(), Y.size()),
      *dM = to_device(0, M.data(), M.size());
    T* dG = nullptr;
    CHECK_CUDA(cudaMalloc(&dG, K * sizeof(T)));
    CHECK_GLMB(Api<T>::gradient()(dX, dM, dY, dG, nullptr, nf, nt, ntasks, nobs, lam, alpha, GLMB_GRAD_REGULARIZE,
                                  nullptr, 0, nullptr));
    CHECK_CUDA(cudaDeviceSynchronize());
    const std::vector<T> g1 = to_host(0, dG, K);

    // the same data in ndev contiguous blocks of observations (ragged split)
    const size_t nd = static_cast<size_t>(ndev);
    std::vector<int64_t> nobs_i(nd);
    std::vector<T*> Xi(nd), Yi(nd), Mi(nd), Gi(nd), Bi(nd);
    std::vector<double*> Li(nd);
    int64_t lo = 0;
    for (int i = 0; i < ndev; ++i) {
        const int64_t hi = i + 1 == ndev ? nobs : lo + nobs / ndev + (i % 2 ? 7 : -5);
        nobs_i[size_t(i)] = hi - lo;
        Xi[size_t(i)] = to_device(i, X.data() + lo * ntasks * nf, size_t((hi - lo) * ntasks * nf));
        Yi[size_t(i)] = to_device(i, Y.data() + lo * ntasks * nt, size_t((hi - lo) * ntasks * nt));
        Mi[size_t(i)] = to_device(i, M.data(), M.size());
        CHECK_CUDA(cudaMalloc(&Gi[size_t(i)], K * sizeof(T)));
        CHECK_CUDA(cudaMalloc(&Bi[size_t(i)], K * sizeof(T)));
        CHECK_CUDA(cudaMalloc(&Li[size_t(i)], size_t(ntasks) * sizeof(double)));
        lo = hi;
    }
    auto constX = std::vector<const T*>(Xi.begin(), Xi.end());
    auto constY = std::vector<const T*>(Yi.begin(), Yi.end());
    auto constM = std::vector<const T*>(Mi.begin(), Mi.end());
    CHECK_GLMB(Api<T>::mg_gradient()(mg, constX.data(), constM.data(), constY.data(), Gi.data(), nobs_i.data(), nf, nt,
                                     ntasks, lam, alpha, GLMB_GRAD_REGULARIZE));
    CHECK_GLMB(glmb_mg_synchronize(mg));
    const std::vector<T> g0 = to_host(0, Gi[0], K);
    bool ok = true;
    for (int i = 1; i < ndev; ++i) {
        const std::vector<T> gi = to_host(i, Gi[size_t(i)], K);
        if (std::memcmp(gi.data(), g0.data(), K * sizeof(T)) != 0) {
            std::printf("FAIL %s %s gradient: device %d differs from device 0\n", mode, Api<T>::name, i);
            ok = false;
        }
    }
    const double e = rel_err(widen(g0), widen(g1), 1e-3);
    std::printf("%s %s %s gradient %lldx%lldx%lldx%lld on %d GPUs: rel err vs one GPU %.3e (bar %.0e)\n",
                e <= Api<T>::tol && ok ? "PASS" : "FAIL", mode, Api<T>::name, (long long)nobs, (long long)ntasks,
                (long long)nf, (long long)nt, ndev, e, Api<T>::tol);
    ok = ok && e <= Api<T>::tol;

    // the sharded fit against the one-GPU fit
    const double l1 = 0.5, l2 = 0.25;
    const int n_power = 20, n_iter = 60;
    const uint64_t fseed = 77;
    T* dB = nullptr;
    double* dL = nullptr;
    CHECK_CUDA(cudaSetDevice(0));
    CHECK_CUDA(cudaMalloc(&dB, K * sizeof(T)));
    CHECK_CUDA(cudaMalloc(&dL, size_t(ntasks) * sizeof(double)));
    CHECK_GLMB(Api<T>::fit()(dX, dY, dB, dL, nf, nt, ntasks, nobs, l1, l2, n_power, n_iter, fseed, nullptr, 0,
                             nullptr));
    CHECK_CUDA(cudaDeviceSynchronize());
    const std::vector<T> b1 = to_host(0, dB, K);
    const std::vector<double> L1 = to_host(0, dL, size_t(ntasks));
    CHECK_GLMB(Api<T>::mg_fit()(mg, constX.data(), constY.data(), Bi.data(), Li.data(), nobs_i.data(), nf, nt, ntasks,
                                l1, l2, n_power, n_iter, fseed));
    CHECK_GLMB(glmb_mg_synchronize(mg));
    const std::vector<T> b0 = to_host(0, Bi[0], K);
    const std::vector<double> L0 = to_host(0, Li[0], size_t(ntasks));
    for (int i = 1; i < ndev; ++i) {
        const std::vector<T> bi = to_host(i, Bi[size_t(i)], K);
        const std::vector<double> Lx = to_host(i, Li[size_t(i)], size_t(ntasks));
        if (std::memcmp(bi.data(), b0.data(), K * sizeof(T)) != 0 ||
            std::memcmp(Lx.data(), L0.data(), size_t(ntasks) * sizeof(double)) != 0) {
            std::printf("FAIL %s %s fit: device %d differs from device 0\n", mode, Api<T>::name, i);
            ok = false;
        }
    }
    const double eb = rel_err(widen(b0), widen(b1), 1e-3), eL = rel_err(L0, L1, 0.0);
    const bool fit_ok = eb <= 10 * Api<T>::tol && eL <= Api<T>::tol;
    std::printf("%s %s %s fit (%d power + %d ISTA) on %d GPUs: beta rel err %.3e, L rel err %.3e\n",
                fit_ok ? "PASS" : "FAIL", mode, Api<T>::name, n_power, n_iter, ndev, eb, eL);
    ok = ok && fit_ok;

    for (int i = 0; i < ndev; ++i) {
        CHECK_CUDA(cudaSetDevice(i));
        cudaFree(Xi[size_t(i)]);
        cudaFree(Yi[size_t(i)]);
        cudaFree(Mi[size_t(i)]);
        cudaFree(Gi[size_t(i)]);
        cudaFree(Bi[size_t(i)]);
        cudaFree(Li[size_t(i)]);
    }
    CHECK_CUDA(cudaSetDevice(0));
    cudaFree(dX);
    cudaFree(dY);
    cudaFree(dM);
    cudaFree(dG);
    cudaFree(dB);
    cudaFree(dL);
    return ok;
}

}  // namespace

int main(int argc, char** argv) {
    const int ndev = argc > 1 ? std::atoi(argv[1]) : 2;
    const std::string which = argc > 2 ? argv[2] : "both";
    int have = 0;
    CHECK_CUDA(cudaGetDeviceCount(&have));
    if (have < ndev) {
        std::printf("SKIP %d GPUs visible, %d asked\n", have, ndev);
        return 0;
    }
    std::vector<int> devs(static_cast<size_t>(ndev));
    for (int i = 0; i < ndev; ++i) devs[size_t(i)] = i;
    bool ok = true;
    for (const char* mode : {"peer", "nccl"}) {
        if (which != "both" && which != mode) continue;
        glmb_mg* mg = nullptr;
        const uint32_t m = std::strcmp(mode, "peer") == 0 ? GLMB_MG_PEER : GLMB_MG_NCCL;
        CHECK_GLMB(glmb_mg_create(ndev, devs.data(), 1 << 16, 5000.0, m, &mg));
        if (glmb_mg_size(mg) != ndev) {
            std::printf("FAIL size\n");
            return 4;
        }
        // the fused rows path (1 task, 1 target), a multi-task rows shape, the float64 tiles path
        ok = run<float>(mg, ndev, mode, Problem{200000, 1, 128, 1}, 1) && ok;
        ok = run<float>(mg, ndev, mode, Problem{30001, 3, 64, 2}, 2) && ok;
        ok = run<double>(mg, ndev, mode, Problem{20000, 2, 96, 3}, 3) && ok;
        ok = run<double>(mg, ndev, mode, Problem{5000, 2, 256, 12}, 4) && ok;
        CHECK_GLMB(glmb_mg_destroy(mg));
    }
    std::printf(ok ? "ALL PASS\n" : "SOME FAILED\n");
    return ok ? 0 : 1;
}
