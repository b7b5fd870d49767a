// glm_tiles.cu -- tiled double-precision GLM gradient for many targets.
//
// For shapes whose per-row work is a small dense contraction (ntargets up
// to 16, nfeatures up to 256, e.g. 64 tasks x 256 features x 16 targets)
// the row-streaming kernel cannot hold nt x nf accumulators per lane.  Here
// a CTA owns one (task, block of observations) and walks it in tiles of
// kTileRows rows, two CTAs per SM (so that one CTA's block barriers overlap
// the other's tensor work).  Both contractions run on the FP64 tensor pipe
// with the 16 x 8 x 16 double MMA (mma.sync m16n8k16 f64: 2048 multiply-adds
// per instruction, eight times the m8n8k4 shape's):
//
//   1. the tile's X rows (nf doubles each) are brought into shared memory by
//      cp.async.bulk copies completing on an mbarrier, into three buffers;
//      a tile's copy is issued two rounds before its step 2 runs;
//   2. Yhat[rows, t] = X_tile . M_task^T: warp w computes the 16 rows x 8
//      targets block (w & 1) over the K quarter (w >> 1), the model's
//      fragments held in registers for the CTA's whole life;
//   3. one thread per (row, target) sums the four K quarters in a fixed
//      order, writes Yhat when asked for and r = yhat - y into shared memory;
//   4. G[t, f] += r^T . X_tile: warp w owns features [32w, 32w + 32) (four
//      16 x 8 blocks over all 16 targets, K = the tile's 16 rows), G held in
//      registers for the CTA's whole block.
//
// The loop is software-pipelined: one round runs step 2 of tile i+1 (four
// MMAs in two dependent chains) and step 4 of tile i (independent MMAs)
// between the same two block barriers, then step 3 of tile i+1, so the
// chains' latency hides behind step 4 and a round has eight MMAs per warp.
//
// X is read from HBM once; yhat and r stay on chip.  The CTA writes one
// double per (t, f) to the partial buffer; glm_finalize_kernel reduces over
// CTAs in a fixed order.  Every wait on an mbarrier is bounded: after
// kWaitLimit polls the thread records an error in the status word and waits
// no more (no further copies are issued), and a kernel after the finalize
// turns that into NaN gradients (no hang).
#include <algorithm>
#include <cstdlib>

#include "glm_common.cuh"
#include "glm_tiles.cuh"

namespace glmb {

namespace {

constexpr int kTileRows = 16;                 // observations per tile (the MMA's M for step 2, K for step 4)
constexpr int kTileThreads = 256;             // 8 warps
constexpr int kCtasPerSm = 2;
constexpr int kMaxF = 256;                    // features per CTA pass
constexpr int kMaxT = 16;                     // targets
constexpr int kBufs = 3;                      // X tile buffers: two copies in flight
constexpr int kMmaK = 16;                     // K of one MMA
constexpr int kKQuarterSteps = kMaxF / 4 / kMmaK;  // MMA steps in a warp's K quarter (4)
constexpr int kXStride = kMaxF + 4;           // padded row stride (doubles): conflict-free fragments
constexpr int kRStride = kMaxT + 4;
constexpr long long kWaitLimit = 1ll << 26;   // mbarrier polls before giving up

struct TilesSmem {
    double X[kBufs][kTileRows][kXStride];
    double D[4][kTileRows][kRStride];  // step 2's four K quarters of X_tile . M^T
    double R[kTileRows][kRStride];     // r = yhat - y (zero outside the data)
    unsigned long long full[kBufs];
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

// D = A(16x16, row) * B(16x8, col) + D on the FP64 tensor pipe.  With
// g = lane / 4, q = lane % 4, the fragments are
//   a[i] = A[g + 8 (i % 2)][q + 4 (i / 2)]   (i < 8)
//   b[i] = B[q + 4 i][g]                      (i < 4)
//   d[i] = D[g + 8 (i / 2)][2 q + i % 2]      (i < 4)
__device__ __forceinline__ void dmma16(double (&d)[4], const double (&a)[8], const double (&b)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, "
        "{%12,%13,%14,%15}, {%0,%1,%2,%3};"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]), "d"(b[0]),
          "d"(b[1]), "d"(b[2]), "d"(b[3]));
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
    const int g = lane >> 2, q = lane & 3;
    const int64_t task = blockIdx.x / a.ctas_per_task;
    const int64_t cta = blockIdx.x - task * a.ctas_per_task;
    const int64_t obs_begin = cta * a.obs_per_cta;
    const int64_t obs_end = min(a.nobs, obs_begin + a.obs_per_cta);
    const int nf = int(a.nf), nt = int(a.nt);
    const int64_t ntasks = a.ntasks;

    // step 2's assignment: targets [8 nb, 8 nb + 8), K quarter kq of the
    // features zero padded to a multiple of 64 (ksteps MMAs of K = 16)
    const int nb = warp & 1, kq = warp >> 1;
    const int kpad = (nf + 63) & ~63;
    const int ksteps = kpad / 64;
    const int kbase = kq * (kpad / 4);
    const bool step2 = nb * 8 < nt;

    // the model's B fragments for this warp's block: M[8 nb + g][kbase + 16 s + q + 4 i]
    double mreg[kKQuarterSteps][4];
#pragma unroll
    for (int s = 0; s < kKQuarterSteps; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = nb * 8 + g, f = kbase + kMmaK * s + q + 4 * i;
            mreg[s][i] = (s < ksteps && t < nt && f < nf) ? a.M[(task * nt + t) * nf + f] : 0.0;
        }

    // X buffers zeroed: padding columns stay zero (they meet zero model
    // coefficients), rows past the end of the data meet r = 0
    for (int i = tid; i < kBufs * kTileRows * kXStride; i += kTileThreads) (&sm.X[0][0][0])[i] = 0.0;
    if (tid == 0) {
#pragma unroll
        for (int b = 0; b < kBufs; ++b) mbar_init(&sm.full[b], 1);
    }
    fence_proxy_async();
    __syncthreads();

    const int ntiles = obs_end > obs_begin ? int((obs_end - obs_begin + kTileRows - 1) / kTileRows) : 0;
    const uint32_t row_bytes = uint32_t(nf) * 8u;

    // Tiles are copied, waited for, and worked on in order, so every index
    // below advances by a fixed step per tile: buffer numbers rotate
    // 0, 1, 2, 0, ..., the copy barriers' parity flips each time the
    // rotation wraps, and row offsets grow by 16 rows.

    // copies: warp 0 issues the next tile (one bulk copy per row) into buffer ib
    bool failed = false;  // this thread's wait on a copy gave up: it waits no more
    int next_issue = 0, ib = 0;
    auto issue_next = [&]() {
        if (next_issue >= ntiles) return;
        if (warp == 0 && !__any_sync(0xffffffffu, failed)) {
            const int64_t first = obs_begin + int64_t(next_issue) * kTileRows;
            const int rows = int(min(int64_t(kTileRows), obs_end - first));
            if (lane == 0) mbar_arrive_expect_tx(&sm.full[ib], uint32_t(rows) * row_bytes);
            __syncwarp();
            if (lane < rows)
                bulk_copy_g2s(&sm.X[ib][lane][0], a.X + ((first + lane) * ntasks + task) * a.nf, row_bytes,
                              &sm.full[ib]);
        }
        ++next_issue;
        ib = ib == kBufs - 1 ? 0 : ib + 1;
    };

    issue_next();
    issue_next();
    issue_next();

    // Every thread waits for a tile's copy itself (no block barrier).  A wait
    // that runs out records the error and the thread goes on without waiting
    // again, so every thread still reaches every block barrier; the result is
    // overwritten with NaN afterwards.
    int wb = 0;
    uint32_t wpar = 0;
    auto wait_next = [&]() {
        if (!failed) {
            long long polls = 0;
            while (!mbar_try_wait(&sm.full[wb], wpar)) {
                if (++polls > kWaitLimit) {
                    failed = true;
                    atomicExch(a.status, 1);
                    break;
                }
            }
        }
        wb = wb == kBufs - 1 ? 0 : wb + 1;
        wpar ^= wb == 0 ? 1u : 0u;
    };

    // step 4's accumulators: G[g + 8 (i / 2)][32 warp + 8 j + 2 q + i % 2]
    double acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0;
    const int nblocks4 = min(4, max(0, (nf - warp * 32 + 7) / 8));  // feature blocks of this warp with data

    // step 3's element: (row, target) of this thread.  Its y is loaded two
    // tiles ahead (Y streams from DRAM; a whole tile of work hides the
    // latency); y and Yhat share the offset ((obs * ntasks + task) * nt + t3).
    const int r3 = tid >> 4, t3 = tid & 15;
    const bool t3_ok = t3 < nt;
    const int rows3 = int(min(int64_t(ntiles) * kTileRows, obs_end - obs_begin)) - r3;  // this row's tiles: 16 t < rows3
    const int64_t off3 = ((obs_begin + r3) * ntasks + task) * a.nt + t3;  // tile 0
    const int64_t step3 = int64_t(kTileRows) * ntasks * a.nt;             // per tile
    int y_tile = 0, r_tile = 0;
    auto load_y_next = [&]() -> double {
        const double v = (a.Y != nullptr && t3_ok && kTileRows * y_tile < rows3) ? a.Y[off3 + y_tile * step3] : 0.0;
        ++y_tile;
        return v;
    };

    // step 2: this warp's K quarter of the 16 x 8 block (rows x targets nb), two chains
    auto step2_mma = [&](int b, double (&d)[2][4]) {
        const double* xs = &sm.X[b][g][kbase + q];
#pragma unroll
        for (int s = 0; s < kKQuarterSteps; ++s) {
            if (s < ksteps) {
                double af[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) af[i] = xs[8 * (i & 1) * kXStride + kMmaK * s + 4 * (i >> 1)];
                dmma16(d[s & 1], af, mreg[s]);
            }
        }
    };
    auto store_d = [&](const double (&d)[2][4]) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sm.D[kq][g + 8 * (i >> 1)][nb * 8 + 2 * q + (i & 1)] = d[0][i] + d[1][i];
    };
    // step 3: r = yhat - y for one (row, target) per thread, quarters summed
    // in a fixed order (tiles in order)
    auto step3_next = [&](double y) {
        const bool in = t3_ok && kTileRows * r_tile < rows3;
        const double yhat = (sm.D[0][r3][t3] + sm.D[1][r3][t3]) + (sm.D[2][r3][t3] + sm.D[3][r3][t3]);
        if (in && a.Yhat != nullptr) a.Yhat[off3 + r_tile * step3] = yhat;
        sm.R[r3][t3] = in ? yhat - y : 0.0;
        ++r_tile;
    };
    // step 4: G[t, f] += sum_rows r[row, t] * x[row, f] over this warp's feature blocks
    auto step4 = [&](int b) {
        const double* xs = &sm.X[b][q][warp * 32 + g];
        double af[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) af[i] = sm.R[q + 4 * (i >> 1)][g + 8 * (i & 1)];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j < nblocks4) {
                double bf[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) bf[i] = xs[4 * i * kXStride + 8 * j];
                dmma16(acc[j], af, bf);
            }
        }
    };

    // Software pipeline over tiles: the first tile's steps 2 and 3 run ahead;
    // then each round issues step 2 of the next tile (a dependent chain) and
    // step 4 of this one (independent MMAs) between the same two barriers, so
    // the chain's latency hides behind step 4.
    int b4 = 0;  // buffer of the tile step 4 works on
    if (ntiles > 0) {
        const double y0 = load_y_next();
        wait_next();
        double d[2][4] = {{0.0, 0.0, 0.0, 0.0}, {0.0, 0.0, 0.0, 0.0}};
        if (step2) step2_mma(0, d);
        store_d(d);
        __syncthreads();
        step3_next(y0);
        __syncthreads();
    }
    double y_cur = load_y_next();  // y of the tile whose residual step 3 forms next
    for (int tile = 0; tile < ntiles; ++tile) {
        const bool more = tile + 1 < ntiles;  // the same in every thread
        const double y_next = load_y_next();
        const int b2 = b4 == kBufs - 1 ? 0 : b4 + 1;
        double d[2][4] = {{0.0, 0.0, 0.0, 0.0}, {0.0, 0.0, 0.0, 0.0}};
        if (more) {
            wait_next();
            if (step2) step2_mma(b2, d);
        }
        step4(b4);
        if (more) store_d(d);
        // every warp is past step 4 of this tile: its X buffer may be refilled
        fence_proxy_async();
        __syncthreads();
        issue_next();  // tile + 3, into buffer b4
        if (more) step3_next(y_cur);
        __syncthreads();
        y_cur = y_next;
        b4 = b2;
    }

    // this CTA's partial: one double per (t, f)
    const int64_t K = int64_t(nt) * nf;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = g + 8 * (i >> 1);
            const int f = warp * 32 + 8 * j + 2 * q + (i & 1);
            if (t < nt && f < nf) a.part[(task * K + int64_t(t) * nf + f) * a.ctas_per_task + cta] = acc[j][i];
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
