// glm_dense.cu -- float32 gradient for dense shapes (many targets x many
// features) on the 5th-generation tensor cores, with 3xTF32 precision.
//
// The gradient splits into two GEMMs per task:
//   GEMM1  R[obs, t] = sum_f X[obs, f] M[t, f] - Y[obs, t]      (K = features)
//   GEMM2  P_s[t, f] = sum_{obs in split s} R[obs, t] X[obs, f]  (K = observations)
// followed by a fixed-order double sum over the splits s and the elastic-net
// finalize.  Both GEMMs run glm_dense_gemm_kernel on CTA pairs (a cluster of
// two CTAs on two SMs) that compute a 256 x 256 output tile together with
// tcgen05.mma.cta_group::2: each CTA stages its own 128 rows of A and its own
// 128 columns of B (with their low parts) into its shared memory -- TMA
// (cp.async.bulk.tensor, swizzled), a three-stage mbarrier ring of 64 KB
// stages -- and holds its 128 rows of the result in its tensor memory (TMEM);
// one thread of the even CTA issues the MMAs for the pair.  Splitting B over
// the pair halves the bytes each SM must bring in per MMA, which pays for
// the deeper ring: with one CTA per tile, two 96 KB stages could not hide
// the L2 latency of the next K block behind the MMAs of the current one.
//
// 3xTF32 (Ootomo & Yokota, 2022): every fp32 operand a is split into two
// tf32 values, hi = a rounded to the nearest tf32 value and lo = a - hi
// (exact in fp32) rounded to the nearest tf32 value (|a - hi - lo| <=
// 2^-22 |a|); each product is hi*hi + hi*lo + lo*hi.  Rounding hi to nearest
// matters: the tensor core reads an fp32 word's high 19 bits, and with that
// truncated hi every lo carries the sign of its a, so the dropped lo*lo term
// is a bias proportional to the product itself -- predictions shrink by
// about 5e-8 of their size, which near a solution (residuals 60x smaller
// than the predictions, summed over 2^20 observations) is several times the
// float rounding of the host algorithm.  With hi to nearest, lo has either
// sign and the dropped term averages out.  The split of M and R is written
// to global memory once (M by a small kernel, R by GEMM1's epilogue) and
// loaded by TMA; each staged X tile is split in shared memory (hi in place,
// lo beside it) by converter warps while the previous stage is multiplied.
//
// Accumulation.  The tensor core rounds each accumulation toward zero, so a
// long accumulation in TMEM drifts towards zero by about half an ulp of the
// running sum per MMA: a bias that follows the sign of the result and, where
// the gradient is a small difference of large terms (near a solution), is far
// larger than fp32 rounding.  So each 32-deep K block is accumulated from
// zero in one of two TMEM buffers (256 columns each) -- its 8 small
// correction products first, then the 4 main ones, so that only 4 roundings
// happen at the block's full magnitude -- and eight epilogue warps add the
// block into fp32 registers (round to nearest) while the tensor core fills
// the other buffer.
//
// Operand majors: GEMM1 reads X and M K-major (features contiguous, 128-byte
// swizzle: one 32-float row per K block); GEMM2 reads R (targets contiguous)
// and X (features contiguous) MN-major, so X is never transposed (MN-major
// 32-bit operands use the 32-byte-chunk variant of the 128-byte swizzle, on
// both the TMA and the descriptor side).
// Pair protocol: each CTA waits for its own TMA copies; its converter warps
// then arrive on the even CTA's `ready` barrier (remote arrive, cluster
// scope), and its drain warps on the even CTA's `acce` barrier; the MMA
// issuer's commits reach both CTAs' `empty`, `accf` and `done` barriers
// (tcgen05.commit multicast).  No TMA copy is multicast.
// Every mbarrier wait is bounded; on expiry the CTA records the failure in a
// status word, skips its remaining work, waits (bounded) for its copies and
// MMAs in flight, meets its peer at the final cluster barrier, frees its
// TMEM and exits, and the reduction kernel turns the status into NaN.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "glm_common.cuh"
#include "glm_dense.cuh"

namespace glmb {

namespace {

constexpr int kBM = 128;       // rows of D per CTA (TMEM lanes); a pair covers 256
constexpr int kBN = 256;       // columns of D (of one TMEM buffer), shared by the pair
constexpr int kBNHalf = kBN / 2;  // columns of B staged by each CTA
constexpr int kBK = 32;        // K per stage and per accumulation block (128 bytes of fp32)
constexpr int kStages = 3;
// Warp roles (16 warps): warp 0 TMA, warp 1 TMEM + MMA issue, warps 2-3 and
// 12-15 form the low parts of the staged X tiles, warps 4-11 (warpgroups 1-2)
// drain TMEM and write the tile -- conversion and drains run side by side.
constexpr int kEpiWarp0 = 4;   // first drain warp
constexpr int kEpiWarps = 8;   // two warps per TMEM lane quarter, one per column half
constexpr int kConvWarps = 6;
constexpr int kThreads = 16 * 32;
// Register split (setmaxnreg): launched at 128 per thread (512 x 128 = 65536);
// warpgroups 0 and 3 drop to 56 and the two drain warpgroups rise to 200,
// which adds up to the same 65536 (per SM sub-partition: 56 + 200 + 200 + 56 = 512 per lane).
constexpr uint32_t kRegsControl = 56, kRegsEpilogue = 200;
static_assert(256 * kRegsControl + 256 * kRegsEpilogue <= kThreads * 128, "register split exceeds the launch");
constexpr int kColsPerThread = kBN / 2;
constexpr uint32_t kTmemCols = 2 * kBN;  // two accumulator buffers
constexpr int kATileBytes = kBM * kBK * 4;  // 16 KB
constexpr int kBTileBytes = kBNHalf * kBK * 4;  // 16 KB
constexpr int kAtomBytes = 32 * kBK * 4;    // MN-major: 32 M/N elements x kBK K-rows
constexpr int kStageBytes = 2 * kATileBytes + 2 * kBTileBytes;
constexpr long long kWaitCycles = 4ll << 30;  // ~2 s at 1.9 GHz
constexpr uint32_t kReadyArrivals = 2 * kConvWarps;  // converter warps of both CTAs
constexpr uint32_t kDrainArrivals = 2 * kEpiWarps;   // drain warps of both CTAs

enum : int { kGemm1 = 1, kGemm2 = 2 };

struct DenseSmem {
    // per stage: A, A lo, B, B lo -- each 1024-byte aligned for the swizzle
    alignas(1024) unsigned char stage[kStages][kStageBytes];
    unsigned long long full[kStages];   // this CTA's TMA -> its converters
    unsigned long long ready[kStages];  // (even CTA) converters of both CTAs -> MMA
    unsigned long long empty[kStages];  // MMAs of the stage retired -> each CTA's TMA
    unsigned long long accf[2];         // K block complete in TMEM buffer b -> each CTA's drainers
    unsigned long long acce[2];         // (even CTA) buffer b drained in both CTAs -> MMA
    unsigned long long done;            // every MMA of the pair retired (teardown)
    uint32_t tmem_base;
    int failed;
};

__device__ __forceinline__ uint32_t saddr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(saddr(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(unsigned long long* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Arrive on the barrier at the same shared-memory offset in CTA `rank` of
// this cluster (default semantics: release at CTA scope).  What the arrival
// publishes is either tensor-core input in this CTA's shared memory, made
// visible to the async proxy by fence.proxy.async beforehand, or the end of
// this CTA's TMEM reads, ordered by tcgen05.fence::before_thread_sync.
// (A release at cluster scope measured 750-1200 cycles per arrival here.)
__device__ __forceinline__ void mbar_arrive_rank(unsigned long long* b, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(saddr(b)), "r"(rank));
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Both CTAs of the pair reach this point (every thread of both).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Bounded wait: false when the clock limit ran out (which sets *failed) or, with
// `failed` given, as soon as another role has failed.  Teardown waits pass
// failed == nullptr and only give up on the limit.
__device__ __forceinline__ bool mbar_wait(unsigned long long* b, uint32_t parity, volatile int* failed) {
    const long long t0 = clock64();
    while (!mbar_test(b, parity)) {
        if (failed != nullptr && *failed) return false;
        if (clock64() - t0 > kWaitCycles) {
            if (failed != nullptr) *failed = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            saddr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(saddr(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 "version 1").
// K-major: one row of kBK fp32 per M/N element -- the 64-byte swizzle
//   (layout 4) for kBK = 16, the 128-byte one (layout 2) for kBK = 32 --
//   8-row groups SBO = 8 rows apart.
// MN-major (layout 1, 128-byte swizzle of 32-byte chunks -- the only MN-major
//   layout the tensor core takes for 32-bit operands): 128 B along M/N
//   (32 fp32) per K-row, 4-row groups SBO = 512 bytes apart, 32-element
//   M/N atoms LBO bytes apart.
constexpr uint32_t kLayoutSW128Base32B = 1;
constexpr uint32_t kLayoutKMajor = kBK == 32 ? 2u : 4u;
constexpr uint32_t kSboKMajor = 8 * kBK * 4;
static_assert(kBK == 16 || kBK == 32, "K block: one 64- or 128-byte swizzle row");
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= uint64_t((addr >> 4) & 0x3FFF);
    d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46;  // descriptor version for sm_100
    d |= uint64_t(layout & 7) << 61;
    return d;
}

// Instruction descriptor of kind::tf32: D f32, A/B tf32, majors, N/8, M/16.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4)                               // D format: f32
           | (2u << 7)                             // A format: tf32
           | (2u << 10)                            // B format: tf32
           | (uint32_t(a_mn_major) << 15)          // A major
           | (uint32_t(b_mn_major) << 16)          // B major
           | (uint32_t(N >> 3) << 17)              // N / 8
           | (uint32_t(M >> 4) << 24);             // M / 16
}

// D[256 x N] (+)= A[256 x 8] B[8 x N] over the pair: rows 0-127 of A and D
// in the even CTA, rows 128-255 in the odd one, B's N columns split in halves
// the same way; descriptors and the TMEM address are offsets valid in both.
__device__ __forceinline__ void umma_tf32_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// One arrival on `bar` in both CTAs of the pair once the MMAs issued so far retire.
__device__ __forceinline__ void umma_commit_pair(unsigned long long* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            saddr(bar)),
        "h"(uint16_t(3))
        : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes; the values
// are valid after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// Waits for this thread's outstanding TMEM loads.  The registers pass through
// the statement so that no use of them is scheduled ahead of the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}
// Orders later uses of r after the preceding volatile statement (a wait).
__device__ __forceinline__ void reg_after(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]));
}

__device__ __forceinline__ float tf32_rn(float a) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(a));
    return __uint_as_float(r);
}
// a ~ hi + lo, both tf32 values, hi rounded to nearest (a - hi is exact in fp32)
__device__ __forceinline__ void tf32_split(float a, float& hi, float& lo) {
    hi = tf32_rn(a);
    lo = tf32_rn(a - hi);
}

// Adds the K block held in TMEM buffer `buf` (this thread's row, its 128
// columns) into sum[], then hands the buffer back to the MMA issuer.
__device__ __forceinline__ bool drain_block(DenseSmem& sm, uint32_t tbase, int blk, float (&sum)[kColsPerThread],
                                            volatile int* failed) {
    const int buf = blk & 1;
    if (!mbar_wait(&sm.accf[buf], uint32_t((blk >> 1) & 1), failed)) return false;
    tc_fence_after();
    // batches of 32 columns: two loads in flight per wait
#pragma unroll
    for (int hb = 0; hb < kColsPerThread / 32; ++hb) {
        uint32_t r[2][16];
#pragma unroll
        for (int j = 0; j < 2; ++j) tmem_ld16(tbase + uint32_t(buf * kBN + 32 * hb + 16 * j), r[j]);
        tmem_wait_ld(r[0]);
        reg_after(r[1]);
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 16; ++i) sum[32 * hb + 16 * j + i] += __uint_as_float(r[j][i]);
    }
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive_rank(&sm.acce[buf], 0);
    return true;
}

struct DenseArgs {
    // Per CTA of a pair:
    // GEMM1: A = X (K-major, box kBK x 1 x 128), B = M / M_lo (K-major, box kBK x 128 x 1)
    // GEMM2: A = R / R_lo (MN-major, box 32 x kBK x 1), B = X (MN-major, box 32 x 1 x kBK)
    int64_t nf, nt, ntasks, nobs, nt_pad;
    int64_t k_begin_step;  // GEMM2: observations per split
    const float* Y;        // GEMM1 epilogue
    float* Yhat;           // GEMM1 epilogue (optional)
    float* R;              // GEMM1 out: Yhat - Y, [task][obs][nt_pad]
    float* R_lo;           // GEMM1 out: low tf32 part of R
    float* P;              // GEMM2 out: [split][task][nt][nf]
    int* status;
};

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    glm_dense_gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapA_lo,
                          const __grid_constant__ CUtensorMap mapB, const __grid_constant__ CUtensorMap mapB_lo,
                          const DenseArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the swizzle needs 1024-byte aligned tiles (same offsets in both CTAs of the pair)
    DenseSmem& sm = *reinterpret_cast<DenseSmem*>(
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023)));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();  // 0: even CTA (issues the MMAs), 1: odd CTA
    const int64_t pair = blockIdx.x >> 1;

    // tile coordinates: m0 = this CTA's 128 rows of D (and of A), n0 = the
    // pair's 256 columns of D, nb0 = the 128 columns of B this CTA stages
    int64_t m0, n0, task, k0, k1;
    if constexpr (MODE == kGemm1) {
        m0 = pair * (2 * kBM) + int64_t(rank) * kBM;  // observations
        n0 = int64_t(blockIdx.y) * kBN;               // targets
        task = blockIdx.z;
        k0 = 0;
        k1 = a.nf;
    } else {
        const int64_t ttiles = (a.nt + 2 * kBM - 1) / (2 * kBM);
        m0 = (pair % ttiles) * (2 * kBM) + int64_t(rank) * kBM;  // targets
        n0 = (pair / ttiles) * kBN;                               // features
        const int64_t split = blockIdx.y;
        task = blockIdx.z;
        k0 = split * a.k_begin_step;
        k1 = min(a.nobs, k0 + a.k_begin_step);
    }
    const int64_t nb0 = n0 + int64_t(rank) * kBNHalf;
    const int nkb = int((k1 - k0 + kBK - 1) / kBK);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.ready[s], kReadyArrivals);
            mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm.accf[b], 1);
            mbar_init(&sm.acce[b], kDrainArrivals);
        }
        mbar_init(&sm.done, 1);
        sm.failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // both CTAs allocate, with the same warp and the same destination offset
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&sm.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers exist before anyone arrives on them
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    volatile int* failed = &sm.failed;

    if (warp < kEpiWarp0 || warp >= kEpiWarp0 + kEpiWarps) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
      if (warp == 0) {
        // ---------------- TMA producer (each CTA: its A rows, its half of B) ----------------
        if (lane == 0) {
            // Every GEMM1 pair reads all of M: pairs start at different K blocks
            // so that they do not all ask the same L2 lines for the same tile
            // at once (measured: GEMM1 8% faster; GEMM2, whose shared R tiles
            // are read by many pairs, was slower with it).  Both CTAs of a pair
            // use the same order; the drains sum whole blocks in that order.
            const int rot =
                MODE == kGemm1 && nkb > 1 ? int((unsigned(pair) * 37u + blockIdx.y * 11u) % unsigned(nkb)) : 0;
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kStages;
                if (kb >= kStages && !mbar_wait(&sm.empty[s], uint32_t((kb / kStages - 1) & 1), failed)) break;
                unsigned char* st = sm.stage[s];
                unsigned char* A = st;
                unsigned char* Alo = st + kATileBytes;
                unsigned char* B = st + 2 * kATileBytes;
                unsigned char* Blo = st + 2 * kATileBytes + kBTileBytes;
                const int kr = kb + rot < nkb ? kb + rot : kb + rot - nkb;
                const int kk = int(k0 + int64_t(kr) * kBK);
                if constexpr (MODE == kGemm1) {
                    mbar_expect_tx(&sm.full[s], kATileBytes + 2 * kBTileBytes);
                    tma_load_3d(A, &mapA, kk, int(task), int(m0), &sm.full[s]);
                    tma_load_3d(B, &mapB, kk, int(nb0), int(task), &sm.full[s]);
                    tma_load_3d(Blo, &mapB_lo, kk, int(nb0), int(task), &sm.full[s]);
                } else {
                    mbar_expect_tx(&sm.full[s], 2 * kATileBytes + kBTileBytes);
                    // R / R_lo: 4 atoms of 32 targets x kBK observations
                    for (int j = 0; j < kBM / 32; ++j) {
                        tma_load_3d(A + j * kAtomBytes, &mapA, int(m0) + 32 * j, kk, int(task), &sm.full[s]);
                        tma_load_3d(Alo + j * kAtomBytes, &mapA_lo, int(m0) + 32 * j, kk, int(task), &sm.full[s]);
                    }
                    // X: 4 atoms of 32 features x kBK observations
                    for (int j = 0; j < kBNHalf / 32; ++j)
                        tma_load_3d(B + j * kAtomBytes, &mapB, int(nb0) + 32 * j, int(task), kk, &sm.full[s]);
                }
                issued = kb + 1;
            }
            // teardown: the copies still in flight land before shared memory is released
            for (int kb = issued > kStages ? issued - kStages : 0; kb < issued; ++kb)
                mbar_wait(&sm.full[kb % kStages], uint32_t((kb / kStages) & 1), nullptr);
        }
      } else if (warp == 1 && lane == 0) {
        if (rank == 0) {
            // ---------------- MMA issuer (even CTA, for the pair) ----------------
            constexpr uint32_t idesc = MODE == kGemm1 ? instr_desc(2 * kBM, kBN, false, false)
                                                      : instr_desc(2 * kBM, kBN, true, true);
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kStages, buf = kb & 1;
                if (kb >= 2 && !mbar_wait(&sm.acce[buf], uint32_t(((kb >> 1) - 1) & 1), failed)) break;
                if (!mbar_wait(&sm.ready[s], uint32_t((kb / kStages) & 1), failed)) break;
                tc_fence_after();
                const uint32_t base = saddr(sm.stage[s]);
                const uint32_t A = base, Alo = base + kATileBytes;
                const uint32_t B = base + 2 * kATileBytes, Blo = B + kBTileBytes;
                const uint32_t d = tmem + uint32_t(buf * kBN);
                uint64_t da[kBK / 8], dal[kBK / 8], db[kBK / 8], dbl[kBK / 8];
#pragma unroll
                for (int k = 0; k < kBK / 8; ++k) {
                    if constexpr (MODE == kGemm1) {
                        // K-major: advance 8 fp32 = 32 bytes along the row per MMA
                        da[k] = smem_desc(A + 32 * k, 16, kSboKMajor, kLayoutKMajor);
                        dal[k] = smem_desc(Alo + 32 * k, 16, kSboKMajor, kLayoutKMajor);
                        db[k] = smem_desc(B + 32 * k, 16, kSboKMajor, kLayoutKMajor);
                        dbl[k] = smem_desc(Blo + 32 * k, 16, kSboKMajor, kLayoutKMajor);
                    } else {
                        // MN-major: advance 8 K-rows (two 512-byte groups) per MMA
                        da[k] = smem_desc(A + 1024 * k, kAtomBytes, 512, kLayoutSW128Base32B);
                        dal[k] = smem_desc(Alo + 1024 * k, kAtomBytes, 512, kLayoutSW128Base32B);
                        db[k] = smem_desc(B + 1024 * k, kAtomBytes, 512, kLayoutSW128Base32B);
                        dbl[k] = smem_desc(Blo + 1024 * k, kAtomBytes, 512, kLayoutSW128Base32B);
                    }
                }
                // the block starts from zero: small correction products first, main products last
#pragma unroll
                for (int k = 0; k < kBK / 8; ++k) {
                    umma_tf32_pair(d, dal[k], db[k], idesc, k > 0 ? 1u : 0u);  // lo * hi
                    umma_tf32_pair(d, da[k], dbl[k], idesc, 1u);               // hi * lo
                }
#pragma unroll
                for (int k = 0; k < kBK / 8; ++k) umma_tf32_pair(d, da[k], db[k], idesc, 1u);  // hi * hi
                umma_commit_pair(&sm.empty[s]);
                umma_commit_pair(&sm.accf[buf]);
            }
            // teardown: every MMA issued has retired (in both CTAs) before TMEM is freed
            umma_commit_pair(&sm.done);
        }
        mbar_wait(&sm.done, 0, nullptr);
      } else if (warp >= 2) {
        // ---------------- converters: low parts of the staged X tiles ----------------
        const int ct = (warp < kEpiWarp0 ? warp - 2 : warp - (kEpiWarp0 + kEpiWarps) + 2) * 32 + lane;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % kStages;
            if (!mbar_wait(&sm.full[s], uint32_t((kb / kStages) & 1), failed)) break;
            unsigned char* st = sm.stage[s];
            float4* src = reinterpret_cast<float4*>(MODE == kGemm1 ? st : st + 2 * kATileBytes);
            float4* dst =
                reinterpret_cast<float4*>(MODE == kGemm1 ? st + kATileBytes : st + 2 * kATileBytes + kBTileBytes);
            constexpr int n4 = (MODE == kGemm1 ? kATileBytes : kBTileBytes) / 16;
#pragma unroll 2
            for (int i = ct; i < n4; i += kConvWarps * 32) {
                const float4 v = src[i];
                float4 h, l;
                tf32_split(v.x, h.x, l.x);
                tf32_split(v.y, h.y, l.y);
                tf32_split(v.z, h.z, l.z);
                tf32_split(v.w, h.w, l.w);
                src[i] = h;  // the swizzled positions are the same for both tiles
                dst[i] = l;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive_rank(&sm.ready[s], 0);
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpilogue));
        // ---------------- TMEM drains, then the tile's epilogue ----------------
        const int ew = warp - kEpiWarp0;  // 0..7
        const int quarter = warp & 3;     // the TMEM lanes (rows of D) this warp may read
        const int half = ew >> 2;         // its 128 columns of D
        const uint32_t tbase = tmem + (uint32_t(32 * quarter) << 16) + uint32_t(half * kColsPerThread);
        float sum[kColsPerThread];
#pragma unroll
        for (int i = 0; i < kColsPerThread; ++i) sum[i] = 0.0f;
        bool ok = true;
        for (int kb = 0; kb < nkb && ok; ++kb) ok = drain_block(sm, tbase, kb, sum, failed);

        const int row = 32 * quarter + lane;
        const int64_t c0 = n0 + int64_t(half) * kColsPerThread;
        if constexpr (MODE == kGemm1) {
            const int64_t obs = m0 + row;
            if (ok && obs < a.nobs) {
                // columns [nt, nt_pad) hold zeros (M is zero-filled there) and are written as such
                const int64_t yrow = (obs * a.ntasks + task) * a.nt;
                float* rrow = a.R + (task * a.nobs + obs) * a.nt_pad;
                float* rlrow = a.R_lo + (task * a.nobs + obs) * a.nt_pad;
#pragma unroll
                for (int i = 0; i < kColsPerThread; i += 4) {
                    const int64_t t = c0 + i;
                    if (t < a.nt_pad) {
                        float r[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const bool in = t + u < a.nt;
                            if (in && a.Yhat != nullptr) a.Yhat[yrow + t + u] = sum[i + u];
                            r[u] = sum[i + u] - (in && a.Y != nullptr ? a.Y[yrow + t + u] : 0.0f);
                        }
                        float4 h, l;
                        tf32_split(r[0], h.x, l.x);
                        tf32_split(r[1], h.y, l.y);
                        tf32_split(r[2], h.z, l.z);
                        tf32_split(r[3], h.w, l.w);
                        *reinterpret_cast<float4*>(rrow + t) = h;
                        *reinterpret_cast<float4*>(rlrow + t) = l;
                    }
                }
            }
        } else {
            const int64_t t = m0 + row;
            if (ok && t < a.nt) {
                float* prow = a.P + ((int64_t(blockIdx.y) * a.ntasks + task) * a.nt + t) * a.nf;
#pragma unroll
                for (int i = 0; i < kColsPerThread; i += 4) {
                    const int64_t f = c0 + i;
                    if (f < a.nf)  // nf is a multiple of 4
                        *reinterpret_cast<float4*>(prow + f) = make_float4(sum[i], sum[i + 1], sum[i + 2], sum[i + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no arrival or MMA operand read targets a CTA that has left
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
    if (tid == 0 && sm.failed) atomicExch(a.status, 1);
}

__global__ void dense_m_split_kernel(const float* __restrict__ M, float* __restrict__ M_hi, float* __restrict__ M_lo,
                                     int64_t n) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        tf32_split(M[i], M_hi[i], M_lo[i]);
}

// grad[e] (or partial_out[e]) from sum over splits of P[s][e], in double, fixed order.
__global__ void dense_reduce_kernel(const float* __restrict__ P, int64_t nsplit, int64_t total,
                                    const float* __restrict__ M, float* __restrict__ grad, double* __restrict__ partial_out,
                                    double lambda, double alpha, int reg, const int* __restrict__ status) {
    const bool bad = *status != 0;
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
        double s = 0.0;
        for (int64_t k = 0; k < nsplit; ++k) s += double(P[k * total + e]);
        if (bad) s = __longlong_as_double(0x7ff8000000000000ll);
        if (partial_out != nullptr) partial_out[e] = s;
        else grad[e] = finalize_value<float>(s, M[e], lambda, alpha, reg != 0);
    }
}

// ---- tensor maps (driver entry point fetched through the runtime) ----------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D fp32 map: dims (innermost first), byte strides of dims 1 and 2, box.
// K-major tiles use the 64- or 128-byte swizzle (one row per kBK floats),
// MN-major tiles the 128-byte swizzle of 32-byte chunks (matching the
// descriptors above).
bool make_map(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
              const uint32_t box[3], bool mn_major) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE,
              mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                       : (kBK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B),
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool dense_f32_supported(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs, const void* X, const void* M) {
    return nf >= 32 && nf % 4 == 0 && nt >= 1 && ntasks >= 1 && nobs >= 1 && ntasks <= 65535 &&
           (reinterpret_cast<uintptr_t>(X) & 15u) == 0 && (reinterpret_cast<uintptr_t>(M) & 15u) == 0 &&
           encode_fn() != nullptr;
}

DensePlan dense_f32_plan(int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs) {
    DensePlan p;
    p.nt_pad = (nt + 3) / 4 * 4;
    const int64_t ttiles = (nt + 2 * kBM - 1) / (2 * kBM), ftiles = (nf + kBN - 1) / kBN;
    // observations per GEMM2 split: enough CTAs (two per 256 x 256 tile) for a few waves
    const int64_t ctas = std::max<int64_t>(1, 2 * ttiles * ftiles * ntasks);
    int64_t splits = std::max<int64_t>(1, (4 * int64_t(sm_count()) + ctas - 1) / ctas);
    int64_t per = (nobs + splits - 1) / splits;
    per = std::min<int64_t>(std::max<int64_t>(per, 4 * kBK), 16384);
    per = (per + kBK - 1) / kBK * kBK;
    p.obs_per_split = per;
    p.nsplit = (nobs + per - 1) / per;
    const size_t total = size_t(ntasks) * nt * nf;
    p.r_bytes = round_up(size_t(ntasks) * nobs * p.nt_pad * 4, 256);
    p.p_bytes = round_up(size_t(p.nsplit) * total * 4, 256);
    p.mlo_bytes = round_up(total * 4, 256);
    p.ws_bytes = 2 * p.r_bytes + p.p_bytes + 2 * p.mlo_bytes + 256;
    return p;
}

int dense_f32_gradient(const DensePlan& p, const float* X, const float* M, const float* Y, float* grad,
                       float* Yhat, double* partial_out, int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,
                       double lambda, double alpha, bool reg, void* ws, cudaStream_t stream) {
    char* w = static_cast<char*>(ws);
    float* R = reinterpret_cast<float*>(w);
    float* R_lo = reinterpret_cast<float*>(w + p.r_bytes);
    float* P = reinterpret_cast<float*>(w + 2 * p.r_bytes);
    float* M_lo = reinterpret_cast<float*>(w + 2 * p.r_bytes + p.p_bytes);
    float* M_hi = reinterpret_cast<float*>(w + 2 * p.r_bytes + p.p_bytes + p.mlo_bytes);
    int* status = reinterpret_cast<int*>(w + 2 * p.r_bytes + p.p_bytes + 2 * p.mlo_bytes);
    const int64_t total = ntasks * nt * nf;
    cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream);
    if (e != cudaSuccess) return int(e);

    dense_m_split_kernel<<<unsigned(std::min<int64_t>(4096, (total + 255) / 256)), 256, 0, stream>>>(M, M_hi, M_lo,
                                                                                                      total);
    count_launch();

    CUtensorMap mX1, mM, mMlo, mR, mRlo, mX2;
    const uint64_t xdims[3] = {uint64_t(nf), uint64_t(ntasks), uint64_t(nobs)};
    const uint64_t xstr[2] = {uint64_t(nf) * 4, uint64_t(nf * ntasks) * 4};
    const uint32_t xbox1[3] = {kBK, 1, kBM}, xbox2[3] = {32, 1, kBK};
    const uint64_t mdims[3] = {uint64_t(nf), uint64_t(nt), uint64_t(ntasks)};
    const uint64_t mstr[2] = {uint64_t(nf) * 4, uint64_t(nf * nt) * 4};
    const uint32_t mbox[3] = {kBK, kBNHalf, 1};
    const uint64_t rdims[3] = {uint64_t(p.nt_pad), uint64_t(nobs), uint64_t(ntasks)};
    const uint64_t rstr[2] = {uint64_t(p.nt_pad) * 4, uint64_t(p.nt_pad * nobs) * 4};
    const uint32_t rbox[3] = {32, kBK, 1};
    if (!make_map(&mX1, X, xdims, xstr, xbox1, false) || !make_map(&mM, M_hi, mdims, mstr, mbox, false) ||
        !make_map(&mMlo, M_lo, mdims, mstr, mbox, false) || !make_map(&mR, R, rdims, rstr, rbox, true) ||
        !make_map(&mRlo, R_lo, rdims, rstr, rbox, true) || !make_map(&mX2, X, xdims, xstr, xbox2, true))
        return GLMB_ERR_UNSUPPORTED;

    const size_t smem = sizeof(DenseSmem) + 1024;
    static std::atomic<uint64_t> attr1{0}, attr2{0};
    if ((e = set_smem_limit_once(attr1, glm_dense_gemm_kernel<kGemm1>, smem)) != cudaSuccess) return int(e);
    if ((e = set_smem_limit_once(attr2, glm_dense_gemm_kernel<kGemm2>, smem)) != cudaSuccess) return int(e);
    DenseArgs args{nf, nt, ntasks, nobs, p.nt_pad, p.obs_per_split, Y, Yhat, R, R_lo, P, status};
    // grids count CTAs: two per pair (the kernel's cluster shape)
    const dim3 g1(unsigned(2 * ((nobs + 2 * kBM - 1) / (2 * kBM))), unsigned((nt + kBN - 1) / kBN), unsigned(ntasks));
    glm_dense_gemm_kernel<kGemm1><<<g1, kThreads, smem, stream>>>(mX1, mX1, mM, mMlo, args);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    const int64_t ttiles = (nt + 2 * kBM - 1) / (2 * kBM), ftiles = (nf + kBN - 1) / kBN;
    const dim3 g2(unsigned(2 * ttiles * ftiles), unsigned(p.nsplit), unsigned(ntasks));
    glm_dense_gemm_kernel<kGemm2><<<g2, kThreads, smem, stream>>>(mR, mRlo, mX2, mX2, args);
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    dense_reduce_kernel<<<unsigned(std::min<int64_t>(4096, (total + 255) / 256)), 256, 0, stream>>>(
        P, p.nsplit, total, M, grad, partial_out, lambda, alpha, reg ? 1 : 0, status);
    count_launch();
    return launch_status();
}

}  // namespace glmb
