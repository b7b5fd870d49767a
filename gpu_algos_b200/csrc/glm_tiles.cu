// glm_tiles.cu -- tiled double-precision GLM gradient for many targets.
//
// For shapes whose per-row work is a small dense contraction (ntargets up
// to 16, nfeatures up to 256, e.g. 64 tasks x 256 features x 16 targets)
// the row-streaming kernel cannot hold nt x nf accumulators per lane.  Here
// a CTA owns one (task, block of observations) and walks it in tiles of
// kTileRows rows, two CTAs per SM (so that one CTA's block barriers overlap
// the other's tensor work):
//
//   1. the tile's X rows (nf doubles each) are brought into shared memory by
//      cp.async.bulk copies completing on an mbarrier, two tiles in flight
//      (the copy of tile i+1 overlaps the arithmetic of tile i);
//   2. Yhat[rows, t] = X_tile . M_task^T on the FP64 tensor pipe
//      (mma.sync m8n8k4 f64): four 8 x 8 output blocks, each computed by two
//      warps over the two halves of K, into shared memory (the two halves are
//      added, and y subtracted, when step 3 reads them);
//   3. G[t, f] += r^T . X_tile, again m8n8k4 f64, G held in registers
//      (16 x 256 doubles over 8 warps) for the CTA's whole block.
//
// X is read from HBM once; yhat and r stay on chip.  The CTA writes one
// double per (t, f) to the partial buffer; glm_finalize_kernel reduces over
// CTAs in a fixed order.  Every wait on an mbarrier is bounded: after
// kWaitLimit polls the CTA records an error in the status word and stops, and
// the host-side finalize turns that into NaN gradients (no hang).
#include <algorithm>
#include <cstdlib>

#include "glm_common.cuh"
#include "glm_tiles.cuh"

namespace glmb {

namespace {

constexpr int kTileRows = 16;                 // observations per tile
constexpr int kTileThreads = 256;             // 8 warps
constexpr int kCtasPerSm = 2;
constexpr int kMaxF = 256;                    // features per CTA pass
constexpr int kMaxT = 16;                     // targets
constexpr int kXStride = kMaxF + 4;           // padded row stride (doubles): conflict-free fragments
constexpr int kRStride = kMaxT + 4;
constexpr long long kWaitLimit = 1ll << 26;   // mbarrier polls before giving up

struct TilesSmem {
    double M[kMaxT][kXStride];
    double X[2][kTileRows][kXStride];
    double D[2][kTileRows][kRStride];  // step 2's two K halves of X_tile . M^T
    double Ys[kTileRows][kRStride];    // the tile's y (zero outside the data)
    unsigned long long full[2];
};
static_assert(kCtasPerSm * (sizeof(TilesSmem) + 1024) <= 228 * 1024, "two CTAs per SM");

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

// true once the phase with the given parity has completed
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D = A(8x4, row) * B(4x8, col) + C on the FP64 tensor pipe.
// Fragments: a = A[lane/4][lane%4], b = B[lane%4][lane/4],
// c/d = C[lane/4][(lane%4)*2 + {0,1}].
__device__ __forceinline__ void dmma(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

struct TilesArgs {
    const double* X;
    const double* M;
    const double* Y;  // NULL: zeros
    double* Yhat;     // NULL: not written
    double* part;     // [task][nt*nf][ctas_per_task]
    int* status;      // set to 1 when a wait gave up
    int64_t nf, nt, ntasks, nobs, obs_per_cta;
    int32_t ctas_per_task;
};

__global__ void __launch_bounds__(kTileThreads, kCtasPerSm) glm_tiles_f64_kernel(const TilesArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    TilesSmem& sm = *reinterpret_cast<TilesSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t task = blockIdx.x / a.ctas_per_task;
    const int64_t cta = blockIdx.x - task * a.ctas_per_task;
    const int64_t obs_begin = cta * a.obs_per_cta;
    const int64_t obs_end = min(a.nobs, obs_begin + a.obs_per_cta);
    const int nf = int(a.nf), nt = int(a.nt);
    const int kpad = (nf + 3) & ~3;  // contraction length of step 2, zero padded
    const int64_t ntasks = a.ntasks;

    // model of this task, zero padded to 16 x 256; X buffers zeroed (padding
    // columns stay zero, rows past the end contribute 0 * 0)
    for (int i = tid; i < kMaxT * kXStride; i += kTileThreads) {
        const int t = i / kXStride, f = i % kXStride;
        sm.M[t][f] = (t < nt && f < nf) ? a.M[(task * nt + t) * nf + f] : 0.0;
    }
    for (int i = tid; i < 2 * kTileRows * kXStride; i += kTileThreads) (&sm.X[0][0][0])[i] = 0.0;
    if (tid == 0) {
        mbar_init(&sm.full[0], 1);
        mbar_init(&sm.full[1], 1);
    }
    fence_proxy_async();
    __syncthreads();

    const int64_t ntiles = obs_end > obs_begin ? (obs_end - obs_begin + kTileRows - 1) / kTileRows : 0;
    const uint32_t row_bytes = uint32_t(nf) * 8u;

    // warp 0 issues the copies of one tile: one bulk copy per row
    auto issue = [&](int64_t tile) {
        if (warp != 0 || tile >= ntiles) return;
        const int b = int(tile & 1);
        const int64_t base = obs_begin + tile * kTileRows;
        const int rows = int(min(int64_t(kTileRows), obs_end - base));
        if (lane == 0) mbar_arrive_expect_tx(&sm.full[b], uint32_t(rows) * row_bytes);
        __syncwarp();
        if (lane < rows) {
            const double* src = a.X + ((base + lane) * ntasks + task) * a.nf;
            bulk_copy_g2s(&sm.X[b][lane][0], src, row_bytes, &sm.full[b]);
        }
    };

    issue(0);
    issue(1);

    // G accumulators: warp w owns features [32w, 32w+32) (four 8-wide tiles)
    // for both 8-target halves.
    double acc[2][4][2];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) acc[mi][ni][0] = acc[mi][ni][1] = 0.0;

    // step 2: warp w computes the 8 x 8 block (rows g1_mt, targets g1_nt)
    // over the K half khalf
    const int g1_mt = warp & 1, g1_nt = (warp >> 1) & 1, khalf = warp >> 2;
    const int ksplit = (kpad / 8) * 4;  // a multiple of 4 (one DMMA step)
    const int k_lo = khalf ? ksplit : 0, k_hi = khalf ? kpad : ksplit;
    const int row2 = g1_mt * 8 + (lane >> 2);  // this lane's row of its block
    bool failed = false;

    // This lane's two y values of a tile (K-half-0 warps own them), loaded one
    // tile ahead: Y streams from DRAM, and a whole tile of work hides its
    // latency where the contraction of one tile alone did not.
    auto load_y = [&](int64_t tile, double (&yv)[2]) {
        const int64_t obs = obs_begin + tile * kTileRows + row2;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int t = g1_nt * 8 + (lane & 3) * 2 + i;
            yv[i] = (khalf == 0 && a.Y != nullptr && tile < ntiles && obs < obs_end && t < nt)
                        ? a.Y[(obs * ntasks + task) * a.nt + t]
                        : 0.0;
        }
    };
    double y_cur[2], y_next[2];
    load_y(0, y_cur);

    for (int64_t tile = 0; tile < ntiles; ++tile) {
        const int b = int(tile & 1);
        load_y(tile + 1, y_next);
        const uint32_t parity = uint32_t((tile >> 1) & 1);
        long long polls = 0;
        while (!mbar_try_wait(&sm.full[b], parity)) {
            if (++polls > kWaitLimit) {
                failed = true;
                break;
            }
        }
        if (__syncthreads_or(failed)) {
            if (tid == 0) atomicExch(a.status, 1);
            return;
        }
        const int64_t base = obs_begin + tile * kTileRows;
        const int64_t obs2 = base + row2;

        // step 2: this warp's K half of an 8 x 8 (rows x targets) block
        {
            double d[2] = {0.0, 0.0};
            if (g1_nt * 8 < nt) {
                // four independent accumulator chains (k mod 16)
                double dk[4][2] = {{0.0, 0.0}, {0.0, 0.0}, {0.0, 0.0}, {0.0, 0.0}};
                const double* xa = &sm.X[b][row2][lane & 3];
                const double* mb = &sm.M[g1_nt * 8 + (lane >> 2)][lane & 3];
                int k0 = k_lo;
                for (; k0 + 16 <= k_hi; k0 += 16) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) dmma(dk[j], xa[k0 + 4 * j], mb[k0 + 4 * j]);
                }
#pragma unroll
                for (int j = 0; j < 3; ++j)
                    if (k0 + 4 * j < k_hi) dmma(dk[j], xa[k0 + 4 * j], mb[k0 + 4 * j]);
#pragma unroll
                for (int i = 0; i < 2; ++i) d[i] = (dk[0][i] + dk[1][i]) + (dk[2][i] + dk[3][i]);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int t = g1_nt * 8 + (lane & 3) * 2 + i;
                const bool in = obs2 < obs_end && t < nt;
                sm.D[khalf][row2][t] = in ? d[i] : 0.0;
                if (khalf == 0) sm.Ys[row2][t] = in ? y_cur[i] : 0.0;
            }
        }
        __syncthreads();

        // predictions, when asked for: one element per thread (16 x 16)
        if (a.Yhat != nullptr) {
            const int r = tid >> 4, t = tid & 15;
            const int64_t obs = base + r;
            if (obs < obs_end && t < nt)
                a.Yhat[(obs * ntasks + task) * a.nt + t] = sm.D[0][r][t] + sm.D[1][r][t];
        }

        // step 3: G[t, f] += sum_rows r[row, t] * x[row, f], r = (D0 + D1) - y
        const int nmt = nt > 8 ? 2 : 1;
#pragma unroll
        for (int k0 = 0; k0 < kTileRows; k0 += 4) {
            const int kr = k0 + (lane & 3);
            double av[2], bv[4];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                const int t = mi * 8 + (lane >> 2);
                av[mi] = (sm.D[0][kr][t] + sm.D[1][kr][t]) - sm.Ys[kr][t];
            }
#pragma unroll
            for (int ni = 0; ni < 4; ++ni) bv[ni] = sm.X[b][kr][warp * 32 + ni * 8 + (lane >> 2)];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                if (mi < nmt) {
#pragma unroll
                    for (int ni = 0; ni < 4; ++ni) dmma(acc[mi][ni], av[mi], bv[ni]);
                }
            }
        }
        __syncthreads();  // all reads of X[b], D and Ys done
        fence_proxy_async();
        issue(tile + 2);
        y_cur[0] = y_next[0];
        y_cur[1] = y_next[1];
    }

    // this CTA's partial: one double per (t, f)
    const int64_t K = int64_t(nt) * nf;
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int t = mi * 8 + (lane >> 2);
                const int f = warp * 32 + ni * 8 + (lane & 3) * 2 + i;
                if (t < nt && f < nf) a.part[(task * K + int64_t(t) * nf + f) * a.ctas_per_task + cta] = acc[mi][ni][i];
            }
}

__global__ void tiles_poison_kernel(const int* status, double* partial_out, double* grad, int64_t n) {
    if (*status == 0) return;
    const double nan = __longlong_as_double(0x7ff8000000000000ll);
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        if (partial_out != nullptr) partial_out[i] = nan;
        if (grad != nullptr) grad[i] = nan;
    }
}

}  // namespace

bool tiles_f64_supported(int64_t nf, int64_t nt, int64_t ntasks, const void* X) {
    return nf > 0 && nf <= kMaxF && (nf % 2) == 0 && nt > 0 && nt <= kMaxT && ntasks > 0 &&
           (reinterpret_cast<uintptr_t>(X) & 15u) == 0;
}

TilesPlan tiles_f64_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {
    TilesPlan p;
    const int64_t sms = int64_t(sm_count()) * kCtasPerSm;  // CTAs per wave
    // enough CTAs for several waves, each with >= 4 tiles
    const int64_t want = std::max<int64_t>(1, (8 * sms + ntasks - 1) / ntasks);
    const int64_t most = std::max<int64_t>(1, nobs / (4 * kTileRows));
    int64_t cpt = std::min(want, most);
    // ... and, among CTA counts per task between want/2 and 2*want, the one
    // whose total fills the last wave best (64 tasks with 2 x 148 CTAs per
    // wave: 37 per task = 8 full waves)
    {
        double best = -1.0;
        const int64_t lo = std::max<int64_t>(1, want / 2), hi = std::min(most, 2 * want);
        for (int64_t c = lo; c <= hi; ++c) {
            const int64_t total = c * ntasks, waves = (total + sms - 1) / sms;
            const double fill = double(total) / double(waves * sms);
            if (fill > best + 1e-9 || (fill > best - 1e-9 && std::llabs(c - want) < std::llabs(cpt - want))) {
                best = fill;
                cpt = c;
            }
        }
    }
    int64_t opc = nobs > 0 ? (nobs + cpt - 1) / cpt : 1;
    opc = (opc + kTileRows - 1) / kTileRows * kTileRows;
    cpt = nobs > 0 ? (nobs + opc - 1) / opc : 0;
    p.ctas_per_task = int32_t(cpt);
    p.obs_per_cta = opc;
    p.part_doubles = size_t(ntasks) * nt * nf * std::max<int64_t>(cpt, 1);
    p.smem_bytes = sizeof(TilesSmem);
    return p;
}

int tiles_f64_launch(const TilesPlan& p, const double* X, const double* M, const double* Y, double* Yhat,
                     double* part, int* status, int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,
                     cudaStream_t stream) {
    if (p.ctas_per_task == 0) return GLMB_OK;
    static std::atomic<uint64_t> attr{0};
    const cudaError_t e = set_smem_limit_once(attr, glm_tiles_f64_kernel, p.smem_bytes);
    if (e != cudaSuccess) return int(e);
    TilesArgs a{X, M, Y, Yhat, part, status, nf, nt, ntasks, nobs, p.obs_per_cta, p.ctas_per_task};
    glm_tiles_f64_kernel<<<unsigned(int64_t(p.ctas_per_task) * ntasks), kTileThreads, p.smem_bytes, stream>>>(a);
    count_launch();
    return launch_status();
}

int tiles_poison(const int* status, double* partial_out, double* grad, int64_t n, cudaStream_t stream) {
    if (n == 0) return GLMB_OK;
    tiles_poison_kernel<<<unsigned(std::min<int64_t>(1024, (n + 255) / 256)), 256, 0, stream>>>(status, partial_out,
                                                                                               grad, n);
    count_launch();
    return launch_status();
}

}  // namespace glmb
