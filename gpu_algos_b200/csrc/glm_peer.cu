// glm_peer.cu -- observation-sharded gradient with the cross-GPU sum done
// over NVLink peer memory inside one kernel.
//
// Every rank owns a "symmetric" buffer (the same layout on each GPU):
//   slots[2][world][max_elems] doubles   (double-buffered by call parity)
//   flags[world][kExMaxBlocks] uint64     (last call number received, per
//                                          sender and per exchange block)
//   ctl[2] uint64                         (this rank's completed calls and
//                                          the exchange blocks' ticket; read
//                                          and written by this rank only)
// A sharded evaluation is two launches per rank:
//   1. the usual CTA-partial kernel over the local observations
//      (glm_rows_kernel / glm_tiles_f64_kernel / the generic pair);
//   2. glm_exchange_kernel.  Its CTAs split the gradient's elements into
//      contiguous chunks and work independently: each sums its elements' CTA
//      partials in a fixed order, stores them into slot [parity][rank] of
//      every peer's buffer (plain P2P stores over NVLink), publishes
//      flag[rank][block] = call number with a system-scope release, waits
//      (bounded) until every sender's flag for its block in its own buffer
//      has reached the call number, sums the world slots in rank order -- so
//      every rank obtains bit-identical results -- and applies the
//      elastic-net finalize (or writes the summed partial for the optimizer).
// Slots alternate with the call parity: a sender can be at most one call
// ahead of a receiver still reading, so two slot sets never collide.  The
// call number lives in device memory (ctl[0]): every block of a call reads
// it when it starts and the last block to finish advances it, so a call
// captured in a CUDA graph and replayed exchanges under a new number each
// time, exactly like a call launched from the host.
//
// Waits are bounded by a clock limit (timeout_ms at group creation): on
// expiry the kernel sets the group's status word, writes NaN outputs and
// returns; the host reads the status with glmb_peer_group_status.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>

#include "glm_common.cuh"
#include "glm_peer.cuh"

struct glmb_peer_group {
    int rank = 0, world = 0, device = 0;
    int64_t max_elems = 0;
    size_t bytes = 0;
    void* buf = nullptr;               // own symmetric buffer (cudaMalloc)
    void* peers[GLMB_PEER_MAX_WORLD];  // peer base pointers (own buf at [rank])
    bool opened[GLMB_PEER_MAX_WORLD];  // pointer came from cudaIpcOpenMemHandle
    void** d_peers = nullptr;          // device copy of peers[]
    int* d_status = nullptr;
    long long timeout_cycles = 0;
    bool connected = false;
};

namespace glmb {

namespace {

constexpr int kExThreads = 256;
constexpr int kExMaxBlocks = 1024;   // flags per sender
// Target chunk: one element per warp.  The first phase (the fixed-order sum of
// a rank's CTA partials, as glm_finalize_kernel does it) is bound by L2
// latency, so elements are spread over warps, not walked by one (8 elements
// per warp cost 30 us per call where one costs 4).  The block count depends on
// the element count alone, so every rank launches the same blocks whatever its
// own partial count.
constexpr int kExElemsPerBlock = kExThreads / 32;
// At most this many partials per element: one thread sums an element's
// partials (already reduced ones: the dense path's single partial), so large
// gradients do not leave 31 lanes of every warp idle.
constexpr int64_t kExThreadSumMax = 32;

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

struct ExArgs {
    const double* part;  // [e][nparts]
    int64_t nparts, total, max_elems;
    void* const* peers;  // device array: base pointer of every rank's buffer
    int rank, world;
    long long timeout_cycles;
    int* status;
    const int* local_status;  // the partial kernel's own status word, or NULL
    double lambda, alpha;
    int reg;
};

__device__ __forceinline__ double* slot_of(void* base, int parity, int sender, int world, int64_t max_elems) {
    return static_cast<double*>(base) + (int64_t(parity) * world + sender) * max_elems;
}
__device__ __forceinline__ uint64_t* flags_of(void* base, int world, int64_t max_elems, int sender, int block) {
    return reinterpret_cast<uint64_t*>(static_cast<double*>(base) + 2 * int64_t(world) * max_elems) +
           int64_t(sender) * kExMaxBlocks + block;
}
// ctl[0]: calls this rank has completed; ctl[1]: blocks of the current call done
__device__ __forceinline__ unsigned long long* ctl_of(void* base, int world, int64_t max_elems) {
    return reinterpret_cast<unsigned long long*>(flags_of(base, world, max_elems, world, 0));
}

// The call number every block of this launch exchanges under (ctl[0] + 1).
__device__ __forceinline__ uint64_t call_epoch(void* own, int world, int64_t max_elems) {
    __shared__ uint64_t s_epoch;
    if (threadIdx.x == 0) s_epoch = __ldcg(ctl_of(own, world, max_elems)) + 1;
    __syncthreads();
    return s_epoch;
}

// Called by every block of the launch once its last access to the buffers
// is issued: the last one to arrive records the call as completed.
__device__ __forceinline__ void call_done(void* own, int world, int64_t max_elems, uint64_t epoch, int nblocks) {
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long* ctl = ctl_of(own, world, max_elems);
        __threadfence();
        if (atomicAdd(&ctl[1], 1ull) == static_cast<unsigned long long>(nblocks - 1)) {
            ctl[1] = 0;
            ctl[0] = epoch;
            __threadfence();
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kExThreads)
    glm_exchange_kernel(const ExArgs a, const T* __restrict__ M, T* __restrict__ grad, double* __restrict__ partial_out) {
    pdl_wait_for_producer();  // the partials are the previous kernel's output
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = kExThreads / 32;
    const int blk = blockIdx.x, nblk = gridDim.x;
    const int64_t chunk = (a.total + nblk - 1) / nblk;
    const int64_t lo = min(a.total, int64_t(blk) * chunk), hi = min(a.total, lo + chunk);
    void* own = a.peers[a.rank];
    const uint64_t epoch = call_epoch(own, a.world, a.max_elems);
    const int parity = int(epoch & 1);
    double* mine = slot_of(own, parity, a.rank, a.world, a.max_elems);

    // 1. this rank's partial for the block's elements: fixed-order sum of the
    // CTA partials, a warp per element when there are many, a thread per
    // element when there are few
    if (a.nparts > kExThreadSumMax) {
        for (int64_t e = lo + warp; e < hi; e += nwarps) {
            double s = 0.0;
            // unrolled: eight independent loads in flight, the additions in the same order
#pragma unroll 8
            for (int64_t c = lane; c < a.nparts; c += 32) s += a.part[e * a.nparts + c];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            if (lane == 0) mine[e] = s;
        }
    } else {
        for (int64_t e = lo + tid; e < hi; e += kExThreads) {
            double s = 0.0;
            for (int64_t c = 0; c < a.nparts; ++c) s += a.part[e * a.nparts + c];
            mine[e] = s;
        }
    }
    __syncthreads();
    // 2. push them into the same slot of every peer's buffer, then raise this
    // block's flag on every rank.  The block barrier orders every thread's
    // stores before the flag writers' system-scope releases (release
    // semantics are cumulative over what the barrier ordered before them),
    // so no thread needs a fence of its own.
    for (int p = 0; p < a.world; ++p) {
        if (p == a.rank) continue;
        double* dst = slot_of(a.peers[p], parity, a.rank, a.world, a.max_elems);
        for (int64_t e = lo + tid; e < hi; e += kExThreads) dst[e] = mine[e];
    }
    __syncthreads();
    if (tid < a.world) st_release_sys(flags_of(a.peers[tid], a.world, a.max_elems, a.rank, blk), epoch);

    // 3. wait until every sender's chunk of this call has arrived (bounded)
    bool failed = false;
    if (tid < a.world) {
        const uint64_t* f = flags_of(own, a.world, a.max_elems, tid, blk);
        const long long t0 = clock64();
        while (ld_acquire_sys(f) < epoch) {
            if (clock64() - t0 > a.timeout_cycles) {
                failed = true;
                break;
            }
            __nanosleep(32);
        }
    }
    if (a.local_status != nullptr && *a.local_status != 0) failed = true;
    failed = __syncthreads_or(failed);
    if (failed) {
        if (tid == 0) atomicExch(a.status, 1);
        const double nan = __longlong_as_double(0x7ff8000000000000ll);
        for (int64_t e = lo + tid; e < hi; e += kExThreads) {
            if (partial_out != nullptr) partial_out[e] = nan;
            else grad[e] = T(nan);
        }
        call_done(own, a.world, a.max_elems, epoch, nblk);
        return;
    }
    // 4. the same rank-ordered sum on every rank, then finalize.  The pollers'
    // acquires happen before the barrier above, so every thread's reads of
    // the slots after it see the senders' stores (read through L2, never a
    // stale L1 line).
    for (int64_t e = lo + tid; e < hi; e += kExThreads) {
        double s = 0.0;
        for (int r = 0; r < a.world; ++r) s += __ldcg(slot_of(own, parity, r, a.world, a.max_elems) + e);
        if (partial_out != nullptr) partial_out[e] = s;
        else grad[e] = finalize_value<T>(s, M[e], a.lambda, a.alpha, a.reg != 0);
    }
    call_done(own, a.world, a.max_elems, epoch, nblk);
}

}  // namespace

int peer_group_create(int rank, int world, int64_t max_elems, double timeout_ms, glmb_peer_group** out,
                      void* handle_out) {
    if (out == nullptr || world < 1 || world > GLMB_PEER_MAX_WORLD || rank < 0 || rank >= world ||
        max_elems < 1 || timeout_ms <= 0)
        return GLMB_ERR_INVALID_VALUE;
    *out = nullptr;
    auto* g = new (std::nothrow) glmb_peer_group();
    if (g == nullptr) return GLMB_ERR_INVALID_VALUE;
    g->rank = rank;
    g->world = world;
    g->max_elems = max_elems;
    for (int i = 0; i < GLMB_PEER_MAX_WORLD; ++i) {
        g->peers[i] = nullptr;
        g->opened[i] = false;
    }
    cudaError_t e = cudaGetDevice(&g->device);
    int clock_khz = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, g->device);
    g->timeout_cycles = static_cast<long long>(timeout_ms * double(clock_khz > 0 ? clock_khz : 2000000));
    g->bytes = size_t(2) * world * max_elems * sizeof(double) + size_t(world) * glmb::kExMaxBlocks * sizeof(uint64_t) +
               2 * sizeof(uint64_t);
    if (e == cudaSuccess) e = cudaMalloc(&g->buf, g->bytes);
    if (e == cudaSuccess) e = cudaMemset(g->buf, 0, g->bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&g->d_peers), sizeof(void*) * GLMB_PEER_MAX_WORLD);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&g->d_status), sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(g->d_status, 0, sizeof(int));
    if (e == cudaSuccess && handle_out != nullptr) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, g->buf);
        if (e == cudaSuccess) std::memcpy(handle_out, &h, sizeof(h));
    }
    if (e != cudaSuccess) {
        peer_group_destroy(g);
        return int(e);
    }
    g->peers[rank] = g->buf;
    *out = g;
    return GLMB_OK;
}

int peer_group_connect(glmb_peer_group* g, const void* handles, void* const* local_ptrs) {
    if (g == nullptr || g->connected || (handles == nullptr && local_ptrs == nullptr)) return GLMB_ERR_INVALID_VALUE;
    for (int p = 0; p < g->world; ++p) {
        if (p == g->rank) continue;
        if (local_ptrs != nullptr) {
            if (local_ptrs[p] == nullptr) return GLMB_ERR_INVALID_VALUE;
            g->peers[p] = local_ptrs[p];
        } else {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const char*>(handles) + size_t(p) * GLMB_PEER_HANDLE_BYTES, sizeof(h));
            void* ptr = nullptr;
            const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) return int(e);
            g->peers[p] = ptr;
            g->opened[p] = true;
        }
    }
    const cudaError_t e = cudaMemcpy(g->d_peers, g->peers, sizeof(void*) * GLMB_PEER_MAX_WORLD, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return int(e);
    g->connected = true;
    return GLMB_OK;
}

int peer_group_status(glmb_peer_group* g, int* status, int reset) {
    if (g == nullptr || status == nullptr) return GLMB_ERR_INVALID_VALUE;
    cudaError_t e = cudaMemcpy(status, g->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && reset) e = cudaMemset(g->d_status, 0, sizeof(int));
    return int(e);
}

int peer_group_destroy(glmb_peer_group* g) {
    if (g == nullptr) return GLMB_OK;
    int st = GLMB_OK;
    for (int p = 0; p < GLMB_PEER_MAX_WORLD; ++p)
        if (g->opened[p]) {
            const cudaError_t e = cudaIpcCloseMemHandle(g->peers[p]);
            if (e != cudaSuccess && st == GLMB_OK) st = int(e);
        }
    if (g->buf) cudaFree(g->buf);
    if (g->d_peers) cudaFree(g->d_peers);
    if (g->d_status) cudaFree(g->d_status);
    delete g;
    return st;
}

void* peer_group_buffer(glmb_peer_group* g) { return g ? g->buf : nullptr; }

template <typename T>
int exchange_launch(glmb_peer_group* g, const double* part, int64_t nparts, int64_t total, const T* M, T* grad,
                    double* partial_out, double lambda, double alpha, bool reg, const int* local_status,
                    cudaStream_t stream) {
    if (g == nullptr || !g->connected) return GLMB_ERR_INVALID_VALUE;
    if (total > g->max_elems) return GLMB_ERR_TOO_LARGE;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != g->device) return GLMB_ERR_INVALID_VALUE;
    ExArgs a{part, nparts, total, g->max_elems, g->d_peers, g->rank, g->world, g->timeout_cycles,
             g->d_status, local_status, lambda, alpha, reg ? 1 : 0};
    // every rank derives the same block count from the same total
    const int nblk = int(std::max<int64_t>(1, std::min<int64_t>(kExMaxBlocks, (total + kExElemsPerBlock - 1) / kExElemsPerBlock)));
    const cudaError_t e = pdl_launch(glm_exchange_kernel<T>, dim3(nblk), dim3(kExThreads), 0, stream, a, M, grad,
                                     partial_out);
    count_launch();
    if (e != cudaSuccess) return int(e);
    return launch_status();
}

template int exchange_launch<float>(glmb_peer_group*, const double*, int64_t, int64_t, const float*, float*, double*,
                                    double, double, bool, const int*, cudaStream_t);
template int exchange_launch<__half>(glmb_peer_group*, const double*, int64_t, int64_t, const __half*, __half*,
                                     double*, double, double, bool, const int*, cudaStream_t);
template int exchange_launch<__nv_bfloat16>(glmb_peer_group*, const double*, int64_t, int64_t, const __nv_bfloat16*,
                                            __nv_bfloat16*, double*, double, double, bool, const int*, cudaStream_t);
template int exchange_launch<double>(glmb_peer_group*, const double*, int64_t, int64_t, const double*, double*,
                                     double*, double, double, bool, const int*, cudaStream_t);

}  // namespace glmb
