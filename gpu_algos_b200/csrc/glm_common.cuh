// glm_common.cuh -- shared device/host helpers of libglm_b200.so (sm_100a).
#pragma once

#include <utility>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <type_traits>

#include "glm_b200.h"

namespace glmb {

constexpr int kWarp = 32;

// Kernel launches made by this library (reported by glmb_launch_count).
void count_launch(int n = 1);
// Records which kernel family the current call used (glmb_last_path).
void set_last_path(const char* path);

// SM count of the current device (cached per device).
int sm_count();

// Status of the last launch, mapped onto the C-ABI status space.
inline int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GLMB_OK : static_cast<int>(e);
}

// ---- storage type <-> arithmetic type --------------------------------------
//
// Acc is the type partial sums are carried in.  float inputs carry partials
// in double (the fused kernels sum short runs in float and spill into
// double), double stays double, half computes in float, integers compute
// modulo 2^bits in the unsigned type of the same (or 32-bit) width.
template <typename T>
struct Arith;
template <>
struct Arith<float> {
    using Acc = double;
    using Dot = float;
};
template <>
struct Arith<double> {
    using Acc = double;
    using Dot = double;
};
template <>
struct Arith<__half> {
    using Acc = float;
    using Dot = float;
};
template <>
struct Arith<__nv_bfloat16> {
    using Acc = float;
    using Dot = float;
};

// The 16-bit floating types: binary16 (__half) and bfloat16.  Both compute
// in float and round to their own format on store.
template <typename T>
inline constexpr bool kHalf16 = std::is_same_v<T, __half> || std::is_same_v<T, __nv_bfloat16>;
__device__ __forceinline__ float half16_to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float half16_to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T float_to_half16(float f) {
    if constexpr (std::is_same_v<T, __half>) return __float2half_rn(f);
    else return __float2bfloat16_rn(f);
}
#define GLMB_INT_ARITH(T, U)   \
    template <>                \
    struct Arith<T> {          \
        using Acc = U;         \
        using Dot = U;         \
    };
GLMB_INT_ARITH(int8_t, uint32_t)
GLMB_INT_ARITH(int16_t, uint32_t)
GLMB_INT_ARITH(int32_t, uint32_t)
GLMB_INT_ARITH(int64_t, uint64_t)
GLMB_INT_ARITH(uint8_t, uint32_t)
GLMB_INT_ARITH(uint16_t, uint32_t)
GLMB_INT_ARITH(uint32_t, uint32_t)
GLMB_INT_ARITH(uint64_t, uint64_t)
#undef GLMB_INT_ARITH

template <typename A, typename T>
__device__ __forceinline__ A to_arith(T v) {
    if constexpr (kHalf16<T>) {
        return static_cast<A>(half16_to_float(v));
    } else {
        return static_cast<A>(v);
    }
}

template <typename T, typename A>
__device__ __forceinline__ T from_arith(A v) {
    if constexpr (kHalf16<T>) {
        return float_to_half16<T>(static_cast<float>(v));
    } else {
        return static_cast<T>(v);
    }
}

// The reference's Number(double) conversion of lambda / alpha.
template <typename T>
__host__ __device__ __forceinline__ T from_double(double d) {
    if constexpr (std::is_same_v<T, __half>) {
        return __double2half(d);
    } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        return __double2bfloat16(d);
    } else {
        return static_cast<T>(d);
    }
}

template <typename T>
__device__ __forceinline__ int sign_of(T v) {
    // include/cuda/cuda_utils.cuh:475-485 of the reference: is_positive /
    // is_negative; unsigned values are never negative, sign(0) = 0.
    if constexpr (kHalf16<T>) {
        const float f = half16_to_float(v);
        return f > 0.f ? 1 : (f < 0.f ? -1 : 0);
    } else if constexpr (std::is_unsigned_v<T>) {
        return v > T(0) ? 1 : 0;
    } else {
        return v > T(0) ? 1 : (v < T(0) ? -1 : 0);
    }
}

template <typename T>
__device__ __forceinline__ bool t_gt0(T v) {
    if constexpr (kHalf16<T>) return half16_to_float(v) > 0.f;
    else return v > T(0);
}
template <typename T>
__device__ __forceinline__ bool t_lt1(T v) {
    if constexpr (kHalf16<T>) return half16_to_float(v) < 1.f;
    else return v < T(1);
}

// Final value of one gradient element from its sum S = sum (yhat - y) * x,
// in the reference's host order (glm_gradient_xyyhat.cuh:839-851):
//   g = 2*S;  if lambda > 0: { if alpha > 0: g += lambda*alpha*sign(M);
//                              if alpha < 1: g += 2*lambda*(1-alpha)*M }
// with every constant formed in the Number type.
template <typename T, typename S>
__device__ __forceinline__ T finalize_value(S sum, T m, double lambda, double alpha, bool reg) {
    using A = typename Arith<T>::Dot;
    A g;
    if constexpr (std::is_floating_point_v<S> && std::is_same_v<A, float>) {
        g = static_cast<float>(2.0 * static_cast<double>(sum));
    } else {
        g = static_cast<A>(A(2) * static_cast<A>(sum));
    }
    if (reg) {
        const T lam_t = from_double<T>(lambda), alp_t = from_double<T>(alpha);
        if (t_gt0(lam_t)) {
            const A lam = to_arith<A>(lam_t), alp = to_arith<A>(alp_t);
            const A two_lambda = A(2) * lam;
            const A one_minus_alpha = A(1) - alp;
            const A two_lambda_one_minus_alpha = two_lambda * one_minus_alpha;
            const A lambda_alpha = lam * alp;
            if (t_gt0(alp_t)) g += lambda_alpha * static_cast<A>(sign_of(m));
            if (t_lt1(alp_t)) g += two_lambda_one_minus_alpha * to_arith<A>(m);
        }
    }
    return from_arith<T>(g);
}

// Sets a kernel's dynamic shared-memory limit once per device: the attribute
// is per device, so a process that drives several GPUs sets it on each
// (`done` holds one bit per device ordinal).
template <typename F>
inline cudaError_t set_smem_limit_once(std::atomic<uint64_t>& done, F* kernel, size_t bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
    return e;
}

// ---- programmatic dependent launch ----------------------------------------
// A kernel that consumes the previous kernel's outputs is launched with
// programmatic stream serialization (pdl_launch) and waits with
// pdl_wait_for_producer() before its first read of them; a producer calls
// pdl_allow_dependents() once it has started, so the consumer's launch
// overlaps the producer's tail.  The consumer is scheduled only after every
// producer CTA has started, so it never takes resources a producer CTA waits for.
__device__ __forceinline__ void pdl_wait_for_producer() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Logistic function 1 / (1 + e^-z) for the logistic link (expf / exp; an
// infinite e^-z gives 0, never NaN).
template <typename D>
__device__ __forceinline__ D sigmoid(D z) {
    if constexpr (std::is_same_v<D, double>) return 1.0 / (1.0 + exp(-z));
    else return 1.0f / (1.0f + expf(-z));
}

// ---- global loads that bypass L1 (X is streamed exactly once) -------------
template <typename T, int VEC>
struct VecLoad;

template <>
struct VecLoad<float, 4> {
    __device__ __forceinline__ static void load(const float* p, float (&v)[4]) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
                     : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                     : "l"(p));
    }
};
template <>
struct VecLoad<double, 2> {
    __device__ __forceinline__ static void load(const double* p, double (&v)[2]) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.f64 {%0,%1}, [%2];"
                     : "=d"(v[0]), "=d"(v[1])
                     : "l"(p));
    }
};
// 16-bit floats (__half, bfloat16): raw 16-bit patterns, element 2i in the
// low half of 32-bit word i.
template <typename T>
__device__ __forceinline__ T half16_from_bits(unsigned short b) {
    if constexpr (std::is_same_v<T, __half>) return __ushort_as_half(b);
    else return __ushort_as_bfloat16(b);
}
template <typename T>
    requires kHalf16<T>
struct VecLoad<T, 8> {
    __device__ __forceinline__ static void load(const T* p, T (&v)[8]) {
        uint32_t r[4];
        asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                     : "l"(p));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = half16_from_bits<T>(static_cast<unsigned short>(r[i] & 0xffffu));
            v[2 * i + 1] = half16_from_bits<T>(static_cast<unsigned short>(r[i] >> 16));
        }
    }
};
template <typename T>
    requires kHalf16<T>
struct VecLoad<T, 4> {
    __device__ __forceinline__ static void load(const T* p, T (&v)[4]) {
        uint32_t r[2];
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "l"(p));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            v[2 * i] = half16_from_bits<T>(static_cast<unsigned short>(r[i] & 0xffffu));
            v[2 * i + 1] = half16_from_bits<T>(static_cast<unsigned short>(r[i] >> 16));
        }
    }
};
template <typename T>
    requires kHalf16<T>
struct VecLoad<T, 2> {
    __device__ __forceinline__ static void load(const T* p, T (&v)[2]) {
        uint32_t r;
        asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
        v[0] = half16_from_bits<T>(static_cast<unsigned short>(r & 0xffffu));
        v[1] = half16_from_bits<T>(static_cast<unsigned short>(r >> 16));
    }
};
template <typename T>
    requires kHalf16<T>
struct VecLoad<T, 1> {
    __device__ __forceinline__ static void load(const T* p, T (&v)[1]) {
        unsigned short r;
        asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
        v[0] = half16_from_bits<T>(r);
    }
};
template <>
struct VecLoad<float, 1> {
    __device__ __forceinline__ static void load(const float* p, float (&v)[1]) {
        asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v[0]) : "l"(p));
    }
};
template <>
struct VecLoad<double, 1> {
    __device__ __forceinline__ static void load(const double* p, double (&v)[1]) {
        asm volatile("ld.global.nc.L1::no_allocate.f64 %0, [%1];" : "=d"(v[0]) : "l"(p));
    }
};

// Scratch for one call: either the caller's workspace or a stream-ordered
// allocation released at the end of the call.
class Scratch {
   public:
    Scratch(void* ws, size_t ws_bytes, size_t need, cudaStream_t s)
        : stream_(s), need_(need) {
        if (need == 0) return;
        if (ws != nullptr) {
            status_ = ws_bytes >= need ? GLMB_OK : GLMB_ERR_WORKSPACE;
            ptr_ = ws;
        } else {
            const cudaError_t e = cudaMallocAsync(&ptr_, need, s);
            status_ = e == cudaSuccess ? GLMB_OK : static_cast<int>(e);
            owned_ = e == cudaSuccess;
        }
    }
    ~Scratch() {
        if (owned_) cudaFreeAsync(ptr_, stream_);
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    int status() const { return status_; }
    template <typename P>
    P* as() const {
        return static_cast<P*>(ptr_);
    }

   private:
    cudaStream_t stream_;
    size_t need_;
    void* ptr_ = nullptr;
    bool owned_ = false;
    int status_ = GLMB_OK;
};

inline size_t round_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

}  // namespace glmb
