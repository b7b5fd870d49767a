// glm_tiles.cu -- tiled double-precision GLM gradient for many targets.
//
// For shapes whose per-row work is a small dense contraction (ntargets up
// to 16, nfeatures up to 256, e.g. 64 tasks x 256 features x 16 targets)
// the row-streaming kernel cannot hold nt x nf accumulators per lane.  Here
// a CTA owns one (task, block of observations) and walks it in tiles of
// kTileRows rows:
//
//   1. the tile's X rows (nf doubles each) are brought into shared memory by
//      cp.async.bulk copies completing on an mbarrier, two tiles in flight
//      (the copy of tile i+1 overlaps the arithmetic of tile i);
//   2. Yhat[rows, t] = X_tile . M_task^T on the FP64 tensor pipe
//      (mma.sync m8n8k4 f64), r = Yhat - y written to shared memory;
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

constexpr int kTileRows = 32;                 // observations per tile
constexpr int kTileThreads = 256;             // 8 warps
constexpr int kMaxF = 256;                    // features per CTA pass
constexpr int kMaxT = 16;                     // targets
constexpr int kXStride = kMaxF + 4;           // padded row stride (doubles): conflict-free fragments
constexpr int kRStride = kMaxT + 4;
constexpr long long kWaitLimit = 1ll << 26;   // mbarrier polls before giving up

struct TilesSmem {
    double M[kMaxT][kXStride];
    double X[2][kTileRows][kXStride];
    double R[kTileRows][kRStride];
    unsigned long long full[2];
};

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

__global__ void __launch_bounds__(kTileThreads, 1) glm_tiles_f64_kernel(const TilesArgs a) {
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

    const int g1_mt = warp & 3;   // step 2: 8-row block of the tile
    const int g1_nt = warp >> 2;  // step 2: 8-target block
    bool failed = false;
    // This warp's B fragments of M for step 2 (targets g1_nt*8.., all of K),
    // held in registers for the CTA's whole block: step 2 then reads only X
    // fragments from shared memory (one 8-byte load per DMMA instead of two).
    double mreg[kMaxF / 4];
    {
        const double* mb = &sm.M[g1_nt * 8 + (lane >> 2)][lane & 3];
#pragma unroll
        for (int k = 0; k < kMaxF / 4; ++k) mreg[k] = mb[4 * k];
    }

    // This lane's two y values of a tile (step 2's residual), loaded one tile
    // ahead: Y streams from DRAM, and a whole tile of work hides its latency
    // where the contraction of one tile alone did not.
    auto load_y = [&](int64_t tile, double (&yv)[2]) {
        const int64_t obs = obs_begin + tile * kTileRows + g1_mt * 8 + (lane >> 2);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int t = g1_nt * 8 + (lane & 3) * 2 + i;
            yv[i] = (a.Y != nullptr && tile < ntiles && obs < obs_end && t < nt) ? a.Y[(obs * ntasks + task) * a.nt + t]
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

        // step 2: yhat for an 8 x 8 (rows x targets) block per warp
        if (g1_nt * 8 < nt) {
            const int row = g1_mt * 8 + (lane >> 2);
            const int64_t obs = base + row;
            const double yv[2] = {y_cur[0], y_cur[1]};
            // four independent accumulator chains over k (k0 mod 16) keep the
            // tensor pipe busy instead of waiting on one dependent chain
            double dk[4][2] = {{0.0, 0.0}, {0.0, 0.0}, {0.0, 0.0}, {0.0, 0.0}};
            const double* xa = &sm.X[b][g1_mt * 8 + (lane >> 2)][lane & 3];
#pragma unroll
            for (int k = 0; k < kMaxF / 4; ++k)
                if (4 * k < kpad) dmma(dk[k & 3], xa[4 * k], mreg[k]);
            double d[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) d[i] = (dk[0][i] + dk[1][i]) + (dk[2][i] + dk[3][i]);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int t = g1_nt * 8 + (lane & 3) * 2 + i;
                double r = 0.0;
                if (obs < obs_end && t < nt) {
                    if (a.Yhat != nullptr) a.Yhat[(obs * ntasks + task) * a.nt + t] = d[i];
                    r = d[i] - yv[i];
                }
                sm.R[row][t] = r;
            }
        } else {
            // targets beyond nt: residual rows are zero
            const int row = g1_mt * 8 + (lane >> 2);
#pragma unroll
            for (int i = 0; i < 2; ++i) sm.R[row][g1_nt * 8 + (lane & 3) * 2 + i] = 0.0;
        }
        __syncthreads();

        // step 3: G[t, f] += sum_rows r[row, t] * x[row, f]
        const int nmt = nt > 8 ? 2 : 1;
#pragma unroll
        for (int k0 = 0; k0 < kTileRows; k0 += 4) {
            const int kr = k0 + (lane & 3);
            double av[2], bv[4];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) av[mi] = sm.R[kr][mi * 8 + (lane >> 2)];
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
        __syncthreads();  // all reads of X[b] and R done
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
    const int64_t sms = sm_count();
    // enough CTAs for several waves of one CTA per SM, each with >= 4 tiles
    const int64_t want = std::max<int64_t>(1, (8 * sms + ntasks - 1) / ntasks);
    const int64_t most = std::max<int64_t>(1, nobs / (4 * kTileRows));
    int64_t cpt = std::min(want, most);
    // ... and, among CTA counts per task between want/2 and 2*want, the one
    // whose total fills the last wave best (64 tasks: 37 per task = 16 full
    // waves of 148, where 19 per task left the 9th wave 78 % empty)
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
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e = cudaFuncSetAttribute(glm_tiles_f64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   int(p.smem_bytes));
        if (e != cudaSuccess) return int(e);
        attr_set = true;
    }
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
