/*
 * glm_b200.h -- C ABI of the B200 (sm_100a) GLM library, libglm_b200.so.
 *
 * Drop-in boundary for the GLM path of alexbaretta/gpu_algos.  In the
 * reference, each kernel class launches its CUDA kernels from a member
 * function `run_device_kernel(..., cudaStream_t)`; in this library the
 * header-only kernel classes (gpu_algos_b200/include/cuda/kernels/glm/)
 * make exactly one call into this ABI instead, and so can any C, C++,
 * ctypes, cgo or JNI caller.
 *
 * Conventions shared by every entry point
 *   - Plain C types only: device pointers, int64_t sizes, doubles, a stream.
 *   - Memory layout is the reference's Tensor3D layout
 *     (include/common/types/tensor3d.hpp:107-112 in the reference):
 *       X     (nfeatures, ntasks, nobs)     X[(obs*ntasks + task)*nf + f]
 *       Y     (ntargets,  ntasks, nobs)     Y[(obs*ntasks + task)*nt + t]
 *       Yhat  same as Y
 *       M     (nfeatures, ntargets, ntasks) M[(task*nt + t)*nf + f]
 *       grad  same as M
 *   - Launches are asynchronous on `stream` (NULL = legacy default stream);
 *     no entry point synchronizes the device or the stream.
 *   - Return value: 0 on success; a cudaError_t value (1..999) when a CUDA
 *     call failed; a GLMB_ERR_* code (>= 1000) for invalid arguments.  No C++
 *     exception crosses this boundary.
 *   - Every output element is overwritten; outputs need no zeroing.
 *   - Scratch memory ("workspace"): entry points that take `workspace` use
 *     it when it is non-NULL and at least the size reported by the matching
 *     *_workspace_size function; with workspace == NULL they obtain scratch
 *     with cudaMallocAsync/cudaFreeAsync on `stream` (stream-ordered, no
 *     synchronisation).
 *   - Types: f16 (__half bits), f32, f64, i8, i16, i32, i64, u8, u16, u32,
 *     u64 -- the eleven `--type` values of the reference mains
 *     (src/cuda/benchmarks/glm/glm_gradient_xyyhat.cu:38-62).  Integer types
 *     compute modulo 2^bits, as the reference's integer kernels do.  Also
 *     bf16 (bfloat16 bits), beyond the reference's type set: float
 *     arithmetic and rounding to bfloat16 on store, as f16 does with
 *     binary16.
 */
#ifndef GLM_B200_H
#define GLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* identical to cudaStream_t */
typedef struct CUstream_st* glmb_stream_t;

#define GLMB_OK 0
#define GLMB_ERR_INVALID_VALUE 1001 /* negative size, NULL pointer for a non-empty tensor */
#define GLMB_ERR_WORKSPACE 1002     /* workspace smaller than required */
#define GLMB_ERR_UNSUPPORTED 1003   /* no device, device is not sm_100, or options the entry point does not offer */
#define GLMB_ERR_TOO_LARGE 1004     /* size beyond a documented limit */
#define GLMB_ERR_COLLECTIVE 1005    /* NCCL could not be loaded, or an NCCL call failed */
#define GLMB_ERR_PEER_TIMEOUT 1006  /* a wait for a peer's partial ran out (that call's outputs are NaN) */

/* gradient flags */
#define GLMB_GRAD_REGULARIZE 0x1u /* add lambda*(alpha*sign(M) + 2*(1-alpha)*M)   */
#define GLMB_GRAD_WRITE_YHAT 0x2u /* also write Yhat = X.M (predictions)           */
#define GLMB_GRAD_Y_ZERO 0x4u     /* Y is all zeros (Y may be NULL)               */
/* Logistic link (half/float/double): with mu = 1/(1 + exp(-X.M)) the
 * gradient is sum_obs (mu - Y) X [+ the elastic-net term], the gradient of
 * the logistic negative log-likelihood, and Yhat (GLMB_GRAD_WRITE_YHAT)
 * receives mu.  The reference's predict kernels carry an unused transform
 * hook for such links (glm_predict_naive.cuh:82-83,550); it applies no link
 * itself.  Not accepted by glmb_gradient_loss_* (whose loss is the squared
 * error) or glmb_gradient_noalloc_f32. */
#define GLMB_GRAD_LOGISTIC 0x8u

/* Library version as an integer (major*10000 + minor*100 + patch). */
int glmb_version(void);

/* Human-readable text for a status code returned by any entry point. */
const char* glmb_status_string(int status);

/* Number of kernels this library has launched in this process. */
uint64_t glmb_launch_count(void);

/* Name of the kernel family the last gradient/predict call on this thread
 * dispatched to ("rows", "generic", ...): diagnostics for tests. */
const char* glmb_last_path(void);

/* ------------------------------------------------------------------------
 * Prediction: Yhat[t, task, obs] = sum_f M[f, t, task] * X[f, task, obs]
 * Replaces Glm_predict_naive_kernel<T>::run_device_kernel
 * (include/cuda/kernels/glm/glm_predict_naive.cuh:525-629).
 * ---------------------------------------------------------------------- */
#define GLMB_DECLARE_PREDICT(SFX, T)                                                    \
    int glmb_predict_##SFX(const T* X, const T* M, T* Yhat, int64_t nfeatures,          \
                           int64_t ntargets, int64_t ntasks, int64_t nobs,              \
                           glmb_stream_t stream);

/* ------------------------------------------------------------------------
 * Gradient of the squared-error loss, fused with the prediction:
 *   grad[f,t,task] = 2 * sum_obs (Yhat - Y)[t,task,obs] * X[f,task,obs]
 *                    [+ lambda*(alpha*sign(M) + 2*(1-alpha)*M)  if GLMB_GRAD_REGULARIZE]
 * With GLMB_GRAD_REGULARIZE this replaces
 *   Glm_gradient_xyyhat_kernel<T>::run_device_kernel
 *   (include/cuda/kernels/glm/glm_gradient_xyyhat.cuh:642-783; the
 *   prediction it stores in `temp` is written when GLMB_GRAD_WRITE_YHAT is set);
 * without it this replaces
 *   Glm_gradient_naive_kernel<T>::run_device_kernel
 *   (include/cuda/kernels/glm/glm_gradient_naive.cuh:342-402).
 * X is read from HBM once; yhat and the residual never leave the chip
 * unless GLMB_GRAD_WRITE_YHAT asks for yhat.
 * ---------------------------------------------------------------------- */
#define GLMB_DECLARE_GRADIENT(SFX, T)                                                   \
    size_t glmb_gradient_workspace_size_##SFX(int64_t nfeatures, int64_t ntargets,      \
                                              int64_t ntasks, int64_t nobs);            \
    int glmb_gradient_##SFX(const T* X, const T* M, const T* Y, T* grad_M, T* Yhat,     \
                            int64_t nfeatures, int64_t ntargets, int64_t ntasks,        \
                            int64_t nobs, double lambda, double alpha, uint32_t flags,  \
                            void* workspace, size_t workspace_bytes,                    \
                            glmb_stream_t stream);

GLMB_DECLARE_PREDICT(f16, uint16_t)
GLMB_DECLARE_PREDICT(bf16, uint16_t)
GLMB_DECLARE_PREDICT(f32, float)
GLMB_DECLARE_PREDICT(f64, double)
GLMB_DECLARE_PREDICT(i8, int8_t)
GLMB_DECLARE_PREDICT(i16, int16_t)
GLMB_DECLARE_PREDICT(i32, int32_t)
GLMB_DECLARE_PREDICT(i64, int64_t)
GLMB_DECLARE_PREDICT(u8, uint8_t)
GLMB_DECLARE_PREDICT(u16, uint16_t)
GLMB_DECLARE_PREDICT(u32, uint32_t)
GLMB_DECLARE_PREDICT(u64, uint64_t)

GLMB_DECLARE_GRADIENT(f16, uint16_t)
GLMB_DECLARE_GRADIENT(bf16, uint16_t)
GLMB_DECLARE_GRADIENT(f32, float)
GLMB_DECLARE_GRADIENT(f64, double)
GLMB_DECLARE_GRADIENT(i8, int8_t)
GLMB_DECLARE_GRADIENT(i16, int16_t)
GLMB_DECLARE_GRADIENT(i32, int32_t)
GLMB_DECLARE_GRADIENT(i64, int64_t)
GLMB_DECLARE_GRADIENT(u8, uint8_t)
GLMB_DECLARE_GRADIENT(u16, uint16_t)
GLMB_DECLARE_GRADIENT(u32, uint32_t)
GLMB_DECLARE_GRADIENT(u64, uint64_t)

/* ------------------------------------------------------------------------
 * Loss (the objective):
 *   loss[0] = sum (Yhat - Y)^2 + lambda*(alpha*sum|M| + (1-alpha)*sum M^2)
 * over every target, task and observation, lambda and alpha taken in T.
 * Replaces Glm_loss_myyhat_kernel<T>::run_device_kernel
 * (include/cuda/kernels/glm/glm_loss_myyhat.cuh:331-363; host definition
 * :365-401).  Y == NULL means zeros.  float/double/half/bfloat16 sum in double,
 * integer types modulo 2^bits (bit-exact with the reference).  Scratch:
 * the gradient workspace of the same shape is enough (or NULL: stream-
 * ordered allocation).  Two launches, one streaming pass over Y and Yhat.
 * ---------------------------------------------------------------------- */
#define GLMB_DECLARE_LOSS(SFX, T)                                                       \
    int glmb_loss_##SFX(const T* M, const T* Y, const T* Yhat, T* loss,                 \
                        int64_t nfeatures, int64_t ntargets, int64_t ntasks,            \
                        int64_t nobs, double lambda, double alpha, void* workspace,     \
                        size_t workspace_bytes, glmb_stream_t stream);

GLMB_DECLARE_LOSS(f16, uint16_t)
GLMB_DECLARE_LOSS(bf16, uint16_t)
GLMB_DECLARE_LOSS(f32, float)
GLMB_DECLARE_LOSS(f64, double)
GLMB_DECLARE_LOSS(i8, int8_t)
GLMB_DECLARE_LOSS(i16, int16_t)
GLMB_DECLARE_LOSS(i32, int32_t)
GLMB_DECLARE_LOSS(i64, int64_t)
GLMB_DECLARE_LOSS(u8, uint8_t)
GLMB_DECLARE_LOSS(u16, uint16_t)
GLMB_DECLARE_LOSS(u32, uint32_t)
GLMB_DECLARE_LOSS(u64, uint64_t)

/* ------------------------------------------------------------------------
 * Gradient and loss from one call (float32/float64): glmb_gradient_* with
 * GLMB_GRAD_WRITE_YHAT (Yhat required) and glmb_loss_* on (M, Y, Yhat) with
 * the same lambda and alpha (the loss always carries the elastic-net term;
 * `flags` governs the gradient's).  X is read once.  Where the row-streaming
 * kernel serves the shape (glmb_last_path() == "rows": at most 8 targets and
 * short rows, up to 1024 float / 512 double features over the targets) it
 * sums the squared residuals in the same pass, in double, and the loss costs
 * no further read of Y or Yhat; other shapes add one read of Y and Yhat.  No single reference call does both;
 * it replaces the reference's xyyhat gradient followed by its loss kernel on
 * the `temp` prediction.
 * ---------------------------------------------------------------------- */
int glmb_gradient_loss_f32(const float* X, const float* M, const float* Y, float* grad_M, float* Yhat,
                           float* loss, int64_t nfeatures, int64_t ntargets, int64_t ntasks, int64_t nobs,
                           double lambda, double alpha, uint32_t flags, void* workspace,
                           size_t workspace_bytes, glmb_stream_t stream);
int glmb_gradient_loss_f64(const double* X, const double* M, const double* Y, double* grad_M,
                           double* Yhat, double* loss, int64_t nfeatures, int64_t ntargets, int64_t ntasks,
                           int64_t nobs, double lambda, double alpha, uint32_t flags, void* workspace,
                           size_t workspace_bytes, glmb_stream_t stream);

/* ------------------------------------------------------------------------
 * Gradient that allocates no device memory (float32).  No counterpart in
 * the reference: it exists for callers that may not allocate -- a host that
 * owns every device buffer and passes a plugin only its inputs and outputs,
 * a fixed device-memory budget, a path that must not wait on the allocator.
 * Same arguments and result as glmb_gradient_f32, minus the workspace: the
 * scratch is a 4 MiB array inside the library, resident on every GPU that
 * loads it until the process exits.  Limits: nfeatures*ntargets*ntasks <=
 * 524288 (else GLMB_ERR_TOO_LARGE), ntargets <= 8 and nfeatures <= 1024
 * (else GLMB_ERR_UNSUPPORTED).  All calls on a device share the array:
 * calls whose kernels overlap on the GPU race, so order them (one stream or
 * events).  The first call on each device looks up the array's address;
 * make it before any stream capture begins.  That address is kept for the
 * life of the process: after cudaDeviceReset on a device, do not call this
 * entry point again in that process.  Throughput: the array holds one double
 * per (task, target, feature) per CTA, so a task gets at most
 * 524288 / (nfeatures*ntargets*ntasks) CTAs; once that falls below the CTAs
 * the single-pass kernel would otherwise use (148 SMs x CTAs per SM, shared
 * by the tasks) the call runs on fewer, longer CTAs and slows accordingly.
 * ---------------------------------------------------------------------- */
int glmb_gradient_noalloc_f32(const float* X, const float* M, const float* Y, float* grad_M,
                              float* Yhat, int64_t nfeatures, int64_t ntargets, int64_t ntasks,
                              int64_t nobs, double lambda, double alpha, uint32_t flags,
                              glmb_stream_t stream);

/* ------------------------------------------------------------------------
 * Sharded evaluation (observations split across GPUs).  The reference is
 * single-GPU (no collective anywhere); these two calls split the gradient
 * around the one exchange step a shard needs:
 *   partial[f,t,task] = sum_{obs in shard} (Yhat - Y)[t,task,obs] * X[f,task,obs]
 * in double, without the factor 2 and without the regularisation term; the
 * caller sums the partials over shards (e.g. an NCCL all-reduce) and
 * finalize applies  grad = 2*partial + lambda*(alpha*sign(M) + 2*(1-alpha)*M)
 * exactly as glmb_gradient_* does on one GPU.
 * ---------------------------------------------------------------------- */
#define GLMB_DECLARE_SHARDED(SFX, T)                                                    \
    int glmb_gradient_partial_##SFX(const T* X, const T* M, const T* Y, double* partial, \
                                    T* Yhat, int64_t nfeatures, int64_t ntargets,       \
                                    int64_t ntasks, int64_t nobs, uint32_t flags,       \
                                    void* workspace, size_t workspace_bytes,            \
                                    glmb_stream_t stream);                              \
    int glmb_gradient_finalize_##SFX(const double* partial, const T* M, T* grad_M,      \
                                     int64_t nfeatures, int64_t ntargets,               \
                                     int64_t ntasks, double lambda, double alpha,       \
                                     uint32_t flags, glmb_stream_t stream);

GLMB_DECLARE_SHARDED(f32, float)
GLMB_DECLARE_SHARDED(f64, double)
GLMB_DECLARE_SHARDED(f16, uint16_t)
GLMB_DECLARE_SHARDED(bf16, uint16_t)

/* ------------------------------------------------------------------------
 * Sharded evaluation with the cross-GPU sum done over NVLink peer memory,
 * inside the library (no collective library on the path).  No counterpart
 * in the reference (single-GPU only).  Each rank creates a group (one
 * device buffer of 2*world*max_elems doubles + world flags, same layout on
 * every rank), exchanges the opaque handles with its peers by any means
 * (e.g. an all-gather of GLMB_PEER_HANDLE_BYTES bytes per rank), and
 * connects.  glmb_gradient_sharded_* then evaluates the full-data gradient
 * from the rank's block of observations: the fused partial kernel, then one
 * exchange kernel that stores the rank's partial into every peer's buffer,
 * waits for all peers (bounded by timeout_ms), sums the partials in rank
 * order -- bit-identical on every rank -- and finalizes.  All ranks must make
 * the same sequence of calls.  A wait that runs out sets the group status
 * (glmb_peer_group_status) and makes that call's outputs NaN.
 * Single-process multi-GPU callers connect with glmb_peer_group_connect_local
 * (peer buffer pointers directly; peer access must be enabled).
 * ---------------------------------------------------------------------- */
#define GLMB_PEER_HANDLE_BYTES 64
#define GLMB_PEER_MAX_WORLD 64
typedef struct glmb_peer_group glmb_peer_group;

int glmb_peer_group_create(int rank, int world, int64_t max_elems, double timeout_ms,
                           glmb_peer_group** group, void* handle_out);
int glmb_peer_group_connect(glmb_peer_group* group, const void* handles /* world x 64 bytes */);
int glmb_peer_group_connect_local(glmb_peer_group* group, void* const* peer_buffers);
void* glmb_peer_group_buffer(glmb_peer_group* group);
int glmb_peer_group_status(glmb_peer_group* group, int* status, int reset);
int glmb_peer_group_destroy(glmb_peer_group* group);

#define GLMB_DECLARE_PEER(SFX, T)                                                       \
    /* grad (or, if partial_out != NULL, the summed double partial) of all ranks' */    \
    int glmb_gradient_sharded_##SFX(const T* X, const T* M, const T* Y, T* grad_M,      \
                                    double* partial_out, T* Yhat, int64_t nfeatures,    \
                                    int64_t ntargets, int64_t ntasks, int64_t nobs,     \
                                    double lambda, double alpha, uint32_t flags,        \
                                    glmb_peer_group* group, void* workspace,            \
                                    size_t workspace_bytes, glmb_stream_t stream);

GLMB_DECLARE_PEER(f32, float)
GLMB_DECLARE_PEER(f64, double)
GLMB_DECLARE_PEER(f16, uint16_t)
GLMB_DECLARE_PEER(bf16, uint16_t)

/* ------------------------------------------------------------------------
 * Elastic-net proximal gradient (ISTA).  No counterpart in the reference,
 * which ships the gradient's elastic-net term
 * (include/cuda/kernels/glm/glm_gradient_xyyhat.cuh:197-211) but no optimizer.
 * Objective: sum (Yhat-Y)^2 + lambda1*|M|_1 + lambda2*|M|^2, i.e. the
 * reference's regularised loss with lambda1 = lambda*alpha and
 * lambda2 = lambda*(1-alpha).
 * ---------------------------------------------------------------------- */
#define GLMB_DECLARE_FIT(SFX, T)                                                        \
    /* beta <- S(beta - grad_smooth*inv_L, l1*inv_L), S = soft threshold */             \
    int glmb_prox_step_##SFX(T* beta, const T* grad_smooth, int64_t n, double inv_L,    \
                             double l1, glmb_stream_t stream);                          \
    /* One fused update from an (all-reduced) partial sum P of the smooth gradient: \
     * g = 2P + 2*lambda2*beta;  beta <- S(beta - g/L[task], lambda1/L[task]),          \
     * L read from device memory (one double per task). */                              \
    int glmb_prox_update_##SFX(const double* partial, T* beta, const double* lipschitz, \
                               int64_t nfeatures, int64_t ntargets, int64_t ntasks,     \
                               double lambda1, double lambda2, glmb_stream_t stream);   \
    /* Power-iteration step from an (all-reduced) partial P = X^T X v:                  \
     * norm[task] = 2*|P_task|;  v_task <- P_task/|P_task|;  and                        \
     * lipschitz[task] = safety*norm[task] + 2*lambda2 (safety = 1.05).                 \
     * v, norm and lipschitz live in device memory. */                                  \
    int glmb_power_step_##SFX(const double* partial, T* v, double* norm,                \
                              double* lipschitz, int64_t nfeatures, int64_t ntasks,     \
                              double lambda2, glmb_stream_t stream);                    \
    /* Seeded start vector of the power iteration (SplitMix64, uniform [-1,1)),         \
     * normalised per task, written to device memory v (nfeatures*ntasks). */            \
    int glmb_power_init_##SFX(T* v, int64_t nfeatures, int64_t ntasks, uint64_t seed,   \
                              glmb_stream_t stream);                                    \
    /* Whole single-GPU fit: n_power power iterations for L, then n_iter ISTA steps     \
     * from beta = 0.  lipschitz (device, ntasks doubles) receives L per task. */       \
    size_t glmb_fit_workspace_size_##SFX(int64_t nfeatures, int64_t ntargets,           \
                                         int64_t ntasks, int64_t nobs);                 \
    int glmb_fit_elastic_net_##SFX(const T* X, const T* Y, T* beta, double* lipschitz,  \
                                   int64_t nfeatures, int64_t ntargets, int64_t ntasks, \
                                   int64_t nobs, double lambda1, double lambda2,        \
                                   int n_power, int n_iter, uint64_t seed,              \
                                   void* workspace, size_t workspace_bytes,             \
                                   glmb_stream_t stream);

GLMB_DECLARE_FIT(f32, float)
GLMB_DECLARE_FIT(f64, double)

/* ------------------------------------------------------------------------
 * Sharded elastic-net fit over a peer-exchange group (one call per rank,
 * every rank with its own block of observations, the same seed and the same
 * arguments otherwise): glmb_fit_elastic_net_* in which every power
 * iteration and ISTA step sums its partial over the group's ranks with the
 * exchange kernel, so every rank ends with the same beta and L.  No
 * counterpart in the reference (single-GPU, no optimizer).  Workspace: the
 * size glmb_fit_workspace_size_* reports for the rank's own nobs.
 * ---------------------------------------------------------------------- */
#define GLMB_DECLARE_SHARDED_FIT(SFX, T)                                                \
    int glmb_fit_elastic_net_sharded_##SFX(const T* X, const T* Y, T* beta,             \
                                           double* lipschitz, int64_t nfeatures,        \
                                           int64_t ntargets, int64_t ntasks,            \
                                           int64_t nobs, double lambda1, double lambda2, \
                                           int n_power, int n_iter, uint64_t seed,      \
                                           glmb_peer_group* group, void* workspace,     \
                                           size_t workspace_bytes, glmb_stream_t stream);

GLMB_DECLARE_SHARDED_FIT(f32, float)
GLMB_DECLARE_SHARDED_FIT(f64, double)

/* ------------------------------------------------------------------------
 * Single-process multi-GPU context, for C and C++ hosts that drive several
 * GPUs from one thread.  It generalises the reference's one-GPU call
 * (Glm_gradient_xyyhat_kernel::run_device_kernel,
 * include/cuda/kernels/glm/glm_gradient_xyyhat.cuh:642) to observations
 * split into one contiguous block per device; the reference has no
 * multi-GPU path, so these calls have no counterpart there.
 *
 * glmb_mg_create     devices[0..ndev) (distinct ordinals), one stream per
 *                    device created here, and the exchange:
 *                      GLMB_MG_PEER  the library's exchange kernel over
 *                                    NVLink peer memory (enables CUDA peer
 *                                    access between the devices);
 *                      GLMB_MG_NCCL  ncclAllReduce, one communicator per
 *                                    device (ncclCommInitAll); NCCL is
 *                                    loaded from libnccl.so.2 at this call
 *                                    (GLMB_ERR_UNSUPPORTED if absent).
 *                    max_elems bounds nfeatures*ntargets*ntasks;
 *                    timeout_ms bounds every peer wait.
 * glmb_mg_gradient   X[i], Y[i]: device i's block (nobs[i] observations,
 *                    Tensor3D layout), M[i]: a copy of the model on device
 *                    i, grad_M[i]: the full-data gradient on device i
 *                    (identical bits on every device).  Flags:
 *                    GLMB_GRAD_REGULARIZE, GLMB_GRAD_Y_ZERO (Y may be NULL),
 *                    GLMB_GRAD_LOGISTIC.
 * glmb_mg_fit_elastic_net   the sharded ISTA fit of glmb_fit_elastic_net_*,
 *                    beta[i] and lipschitz[i] (ntasks doubles) on device i.
 * Calls are asynchronous on the context's streams (glmb_mg_stream) and
 * restore the caller's current device; glmb_mg_synchronize waits for all
 * devices and returns GLMB_ERR_PEER_TIMEOUT if an exchange wait ran out.
 * A context is used by one host thread at a time.
 * ---------------------------------------------------------------------- */
#define GLMB_MG_MAX_DEVICES 64
#define GLMB_MG_PEER 0u
#define GLMB_MG_NCCL 1u
typedef struct glmb_mg glmb_mg;

int glmb_mg_create(int ndev, const int* devices, int64_t max_elems, double timeout_ms, uint32_t mode,
                   glmb_mg** mg);
int glmb_mg_destroy(glmb_mg* mg);
int glmb_mg_size(glmb_mg* mg);
int glmb_mg_stream(glmb_mg* mg, int i, glmb_stream_t* stream);
int glmb_mg_synchronize(glmb_mg* mg);

#define GLMB_DECLARE_MG(SFX, T)                                                         \
    int glmb_mg_gradient_##SFX(glmb_mg* mg, const T* const* X, const T* const* M,       \
                               const T* const* Y, T* const* grad_M, const int64_t* nobs, \
                               int64_t nfeatures, int64_t ntargets, int64_t ntasks,     \
                               double lambda, double alpha, uint32_t flags);            \
    int glmb_mg_fit_elastic_net_##SFX(glmb_mg* mg, const T* const* X, const T* const* Y, \
                                      T* const* beta, double* const* lipschitz,         \
                                      const int64_t* nobs, int64_t nfeatures,           \
                                      int64_t ntargets, int64_t ntasks, double lambda1, \
                                      double lambda2, int n_power, int n_iter,          \
                                      uint64_t seed);

GLMB_DECLARE_MG(f32, float)
GLMB_DECLARE_MG(f64, double)

#ifdef __cplusplus
}
#endif
#endif /* GLM_B200_H */
