/*
 * glm_oracle.c -- CPU restatement of the reference's GLM host path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker); see glm_oracle.h for the list of
 * reference functions restated here and for how the restatement is pinned.
 *
 * Arithmetic follows the reference's `Number` type: float and double
 * compute in their own precision, integer types compute modulo 2^bits (the
 * reference's Eigen products run in the integer type itself, which wraps;
 * wrapping arithmetic is a ring homomorphism, so any summation order gives
 * the same bits), half computes in float and rounds to binary16 on store.
 * bfloat16 (not a type of the reference) is treated like half: float
 * arithmetic, rounded to bfloat16 on store.
 *
 * Summation order.  The reference's product 2*(M*X^T - Y^T)*X
 * (glm_gradient_xyyhat.cuh:839) is an Eigen GEMM, whose depth (obs) loop is
 * split into panels: each panel is accumulated sequentially in registers and
 * then added into the result.  The restatement keeps that shape: obs are cut
 * into panels of ORACLE_KC rows, each panel's products are summed
 * sequentially, panel sums are added into one of at most ORACLE_MAX_CHUNKS
 * chunk accumulators (each a contiguous run of panels), and the chunk
 * accumulators are added in chunk order.  The result does not depend on the
 * number of threads.  Dot products over features use eight interleaved
 * partial sums combined as a tree, the shape of Eigen's packet reduction
 * (glm_predict_naive.cuh:642 calls Eigen's dot).
 */
#include "glm_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_KC 256
#define ORACLE_FT 512 /* features per tile of the accumulation loop (cache blocking only) */
#define ORACLE_MAX_CHUNKS 64
#define ORACLE_POWER_SAFETY 1.05

static int g_threads = 0;

void oracle_set_threads(int nthreads) { g_threads = nthreads; }

int oracle_get_threads(void) {
    return g_threads > 0 ? g_threads : omp_get_max_threads();
}

/* Rows of X in a cache group: about 128 KB of row data, 1 to ORACLE_KC rows
 * (cache blocking only; no result depends on it). */
static inline int64_t oracle_rows_per_group(int64_t row_bytes) {
    int64_t r = row_bytes > 0 ? (int64_t)(131072 / row_bytes) : ORACLE_KC;
    if (r < 1) r = 1;
    return r < ORACLE_KC ? r : ORACLE_KC;
}

/* ---- binary16 helpers (gcc _Float16, round-to-nearest-even) ---- */
static inline float h2f(uint16_t h) {
    _Float16 x;
    memcpy(&x, &h, sizeof(x));
    return (float)x;
}
static inline uint16_t f2h(float f) {
    _Float16 x = (_Float16)f;
    uint16_t h;
    memcpy(&h, &x, sizeof(h));
    return h;
}
/* the reference's Number(double) for half: one rounding from double */
static inline uint16_t d2h(double d) {
    _Float16 x = (_Float16)d;
    uint16_t h;
    memcpy(&h, &x, sizeof(h));
    return h;
}

/* ---- bfloat16 helpers (bit operations, round-to-nearest-even) ----
 * bfloat16 is the high half of a binary32: widening is a shift; narrowing
 * adds 0x7fff plus the kept LSB (ties to even) and keeps the high half,
 * NaNs stay quiet NaNs.  From double the value is first narrowed to float
 * with round-to-odd (truncate, set the LSB when inexact), which makes the
 * second rounding to 8 significant bits equal to one direct rounding. */
static inline float b2f(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
}
static inline uint16_t f2b(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof(u));
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline uint16_t d2b(double d) {
    if (d != d) return f2b((float)d);
    float t = (float)d;
    if ((double)t != d) {
        if (fabs((double)t) > fabs(d)) t = nextafterf(t, 0.0f);
        uint32_t u;
        memcpy(&u, &t, sizeof(u));
        u |= 1u;
        memcpy(&t, &u, sizeof(t));
    }
    return f2b(t);
}

/* ---- per-type load (T -> A), store (A -> T), from-double and sign ---- */
#define LD_plain(A, v) ((A)(v))
#define ST_plain(T, a) ((T)(a))

/* sign as in cuda_utils.cuh:475-485: +1 if > 0, -1 if < 0, else 0 */
#define SIGN_SIGNED(v) (((v) > 0) ? 1 : (((v) < 0) ? -1 : 0))
#define SIGN_UNSIGNED(v) (((v) > 0) ? 1 : 0)

/*
 * ORACLE_DEFINE generates predict / gradient / loss for one type.
 *   T      storage type            A      arithmetic type
 *   LD(v)  T -> A                   ST(a)  A -> T
 *   FROMD(d) double -> T (the reference's Number(double) conversion)
 *   TGT0(v) / TLT0(v) / TLT1(v)   comparisons of a T value with 0 and 1
 *   SGN(v) sign of a T value as int, ABS(v) |v| in A
 */
#define ORACLE_DEFINE(SFX, T, A, LD, ST, FROMD, TGT0, TLT0, TLT1, SGN, ABS)                 \
    static inline A dot_##SFX(const T* x, const T* m, int64_t n) {                          \
        A p0 = 0, p1 = 0, p2 = 0, p3 = 0, p4 = 0, p5 = 0, p6 = 0, p7 = 0;                   \
        int64_t f = 0;                                                                      \
        for (; f + 8 <= n; f += 8) {                                                        \
            p0 += LD(x[f + 0]) * LD(m[f + 0]);                                              \
            p1 += LD(x[f + 1]) * LD(m[f + 1]);                                              \
            p2 += LD(x[f + 2]) * LD(m[f + 2]);                                              \
            p3 += LD(x[f + 3]) * LD(m[f + 3]);                                              \
            p4 += LD(x[f + 4]) * LD(m[f + 4]);                                              \
            p5 += LD(x[f + 5]) * LD(m[f + 5]);                                              \
            p6 += LD(x[f + 6]) * LD(m[f + 6]);                                              \
            p7 += LD(x[f + 7]) * LD(m[f + 7]);                                              \
        }                                                                                   \
        A s = (A)(((A)(p0 + p1) + (A)(p2 + p3)) + ((A)(p4 + p5) + (A)(p6 + p7)));           \
        for (; f < n; ++f) s += LD(x[f]) * LD(m[f]);                                        \
        return s;                                                                           \
    }                                                                                       \
                                                                                            \
    void oracle_glm_predict_##SFX(const T* X, const T* M, T* Yhat, int64_t nf, int64_t nt,  \
                                  int64_t ntasks, int64_t nobs) {                           \
        const int nth = oracle_get_threads();                                               \
        _Pragma("omp parallel for num_threads(nth) schedule(static)")                       \
        for (int64_t obs = 0; obs < nobs; ++obs) {                                          \
            for (int64_t task = 0; task < ntasks; ++task) {                                 \
                const T* x = X + (obs * ntasks + task) * nf;                                \
                for (int64_t t = 0; t < nt; ++t) {                                          \
                    const T* m = M + (task * nt + t) * nf;                                  \
                    Yhat[(obs * ntasks + task) * nt + t] = ST(dot_##SFX(x, m, nf));         \
                }                                                                           \
            }                                                                               \
        }                                                                                   \
    }                                                                                       \
                                                                                            \
    void oracle_glm_gradient_##SFX(const T* X, const T* M, const T* Y, T* grad, int64_t nf, \
                                   int64_t nt, int64_t ntasks, int64_t nobs, double lambda, \
                                   double alpha, int with_reg) {                            \
        const int64_t K = nt * nf;                                                          \
        if (K == 0) return;                                                                 \
        const int64_t nblocks = (nobs + ORACLE_KC - 1) / ORACLE_KC;                         \
        int64_t nchunks = nblocks < ORACLE_MAX_CHUNKS ? nblocks : ORACLE_MAX_CHUNKS;        \
        if (nchunks < 1) nchunks = 1;                                                       \
        while (nchunks > 1 && (double)nchunks * (double)K * sizeof(A) > 512e6) nchunks /= 2; \
        A* part = (A*)calloc((size_t)(nchunks * K), sizeof(A));                             \
        const int nth = oracle_get_threads();                                               \
        const int64_t sub = oracle_rows_per_group(nf * (int64_t)sizeof(T));                 \
        for (int64_t task = 0; task < ntasks; ++task) {                                     \
            const T* Mt = M + task * K;                                                     \
            _Pragma("omp parallel for num_threads(nth) schedule(dynamic, 1)")               \
            for (int64_t c = 0; c < nchunks; ++c) {                                         \
                A* acc = part + c * K;                                                      \
                A* tmp = (A*)malloc((size_t)K * sizeof(A));                                 \
                A* e = (A*)malloc((size_t)(ORACLE_KC * nt) * sizeof(A));                    \
                for (int64_t k = 0; k < K; ++k) acc[k] = 0;                                 \
                const int64_t b0 = c * nblocks / nchunks, b1 = (c + 1) * nblocks / nchunks; \
                for (int64_t b = b0; b < b1; ++b) {                                         \
                    for (int64_t k = 0; k < K; ++k) tmp[k] = 0;                             \
                    const int64_t o0 = b * ORACLE_KC;                                       \
                    const int64_t o1 = o0 + ORACLE_KC < nobs ? o0 + ORACLE_KC : nobs;       \
                    /* residuals of the panel's rows: the panel's (M*X^T - Y^T) block, */   \
                    /* taken in row groups of about 128 KB so that the rows of X and    */   \
                    /* M a group uses stay cached (each dot product as above)           */   \
                    for (int64_t s0 = o0; s0 < o1; s0 += sub) {                             \
                        const int64_t s1 = s0 + sub < o1 ? s0 + sub : o1;                   \
                        for (int64_t t = 0; t < nt; ++t) {                                  \
                            for (int64_t obs = s0; obs < s1; ++obs) {                       \
                                const T* x = X + (obs * ntasks + task) * nf;                \
                                const A yv = Y ? LD(Y[(obs * ntasks + task) * nt + t]) : (A)0; \
                                e[(obs - o0) * nt + t] = dot_##SFX(x, Mt + t * nf, nf) - yv; \
                            }                                                               \
                        }                                                                   \
                    }                                                                       \
                    /* tmp[t][f] += e[obs][t] * x[obs][f], rows in ascending order for  */  \
                    /* every element; features in tiles so that tmp's rows stay cached */   \
                    for (int64_t f0 = 0; f0 < nf; f0 += ORACLE_FT) {                        \
                        const int64_t f1 = f0 + ORACLE_FT < nf ? f0 + ORACLE_FT : nf;       \
                        for (int64_t t = 0; t < nt; ++t) {                                  \
                            A* row = tmp + t * nf;                                          \
                            for (int64_t obs = o0; obs < o1; ++obs) {                       \
                                const T* x = X + (obs * ntasks + task) * nf;                \
                                const A et = e[(obs - o0) * nt + t];                        \
                                for (int64_t f = f0; f < f1; ++f) row[f] += et * LD(x[f]);  \
                            }                                                               \
                        }                                                                   \
                    }                                                                       \
                    for (int64_t k = 0; k < K; ++k) acc[k] += tmp[k];                       \
                }                                                                           \
                free(tmp);                                                                  \
                free(e);                                                                    \
            }                                                                               \
            const T lam_t = FROMD(lambda), alp_t = FROMD(alpha);                            \
            const A lam = LD(lam_t), alp = LD(alp_t);                                       \
            const A two_lambda = (A)2 * lam;                                                \
            const A one_minus_alpha = (A)1 - alp;                                           \
            const A two_lambda_one_minus_alpha = two_lambda * one_minus_alpha;              \
            const A lambda_alpha = lam * alp;                                               \
            for (int64_t k = 0; k < K; ++k) {                                               \
                A s = 0;                                                                    \
                for (int64_t c = 0; c < nchunks; ++c) s += part[c * K + k];                 \
                A g = (A)2 * s;                                                             \
                if (with_reg && TGT0(lam_t)) {                                              \
                    const T mv = Mt[k];                                                     \
                    if (TGT0(alp_t)) g += lambda_alpha * (A)SGN(mv);                        \
                    if (TLT1(alp_t)) g += two_lambda_one_minus_alpha * LD(mv);              \
                }                                                                           \
                grad[task * K + k] = ST(g);                                                 \
            }                                                                               \
        }                                                                                   \
        free(part);                                                                         \
    }                                                                                       \
                                                                                            \
    void oracle_glm_loss_##SFX(const T* M, const T* Y, const T* Yhat, T* loss, int64_t nf,  \
                               int64_t nt, int64_t ntasks, int64_t nobs, double lambda,     \
                               double alpha) {                                              \
        const int64_t size_Y = nt * ntasks * nobs, size_M = nf * nt * ntasks;               \
        A error_loss = 0;                                                                   \
        for (int64_t i = 0; i < size_Y; ++i) {                                              \
            const A err = LD(Yhat[i]) - LD(Y[i]);                                           \
            error_loss += err * err;                                                        \
        }                                                                                   \
        A l1_loss = 0, l2_loss = 0;                                                         \
        for (int64_t i = 0; i < size_M; ++i) l1_loss += ABS(M[i]);                          \
        for (int64_t i = 0; i < size_M; ++i) l2_loss += LD(M[i]) * LD(M[i]);                \
        const A lam = LD(FROMD(lambda)), alp = LD(FROMD(alpha));                            \
        const A reg = lam * (alp * l1_loss + ((A)1 - alp) * l2_loss);                       \
        loss[0] = ST(error_loss + reg);                                                     \
    }                                                                                       \
    typedef int oracle_define_##SFX##_done

/* float / double */
#define LD_F(v) ((float)(v))
#define ST_F(a) ((float)(a))
#define FROMD_F(d) ((float)(d))
#define LD_D(v) ((double)(v))
#define ST_D(a) ((double)(a))
#define FROMD_D(d) ((double)(d))
#define GT0(v) ((v) > 0)
#define LT0(v) ((v) < 0)
#define LT1(v) ((v) < 1)
#define ABS_F(v) fabsf((float)(v))
#define ABS_D(v) fabs((double)(v))

ORACLE_DEFINE(f32, float, float, LD_F, ST_F, FROMD_F, GT0, LT0, LT1, SIGN_SIGNED, ABS_F);
ORACLE_DEFINE(f64, double, double, LD_D, ST_D, FROMD_D, GT0, LT0, LT1, SIGN_SIGNED, ABS_D);

/* half: uint16_t bit patterns, float arithmetic */
#define LD_H(v) h2f(v)
#define ST_H(a) f2h((float)(a))
#define FROMD_H(d) d2h(d)
#define HGT0(v) (h2f(v) > 0.0f)
#define HLT0(v) (h2f(v) < 0.0f)
#define HLT1(v) (h2f(v) < 1.0f)
#define HSIGN(v) ((h2f(v) > 0.0f) ? 1 : ((h2f(v) < 0.0f) ? -1 : 0))
#define ABS_H(v) fabsf(h2f(v))
ORACLE_DEFINE(f16, uint16_t, float, LD_H, ST_H, FROMD_H, HGT0, HLT0, HLT1, HSIGN, ABS_H);

/* bfloat16: uint16_t bit patterns, float arithmetic */
#define LD_B(v) b2f(v)
#define ST_B(a) f2b((float)(a))
#define FROMD_B(d) d2b(d)
#define BGT0(v) (b2f(v) > 0.0f)
#define BLT0(v) (b2f(v) < 0.0f)
#define BLT1(v) (b2f(v) < 1.0f)
#define BSIGN(v) ((b2f(v) > 0.0f) ? 1 : ((b2f(v) < 0.0f) ? -1 : 0))
#define ABS_B(v) fabsf(b2f(v))
ORACLE_DEFINE(bf16, uint16_t, float, LD_B, ST_B, FROMD_B, BGT0, BLT0, BLT1, BSIGN, ABS_B);

/* integers: arithmetic modulo 2^32 (types up to 32 bits) or 2^64 */
#define INT_FROMD(T) (T)
#define ABS_SI(A, v) ((A)((v) < 0 ? -(A)(v) : (A)(v)))
#define LD_U32(v) ((uint32_t)(v))
#define LD_U64(v) ((uint64_t)(v))
#define ABS_I8(v) ((uint32_t)((v) < 0 ? (uint32_t)0 - (uint32_t)(v) : (uint32_t)(v)))
#define ABS_I64(v) ((uint64_t)((v) < 0 ? (uint64_t)0 - (uint64_t)(v) : (uint64_t)(v)))
#define ABS_U32(v) ((uint32_t)(v))
#define ABS_U64(v) ((uint64_t)(v))

#define ST_I8(a) ((int8_t)(a))
#define ST_I16(a) ((int16_t)(a))
#define ST_I32(a) ((int32_t)(a))
#define ST_I64(a) ((int64_t)(a))
#define ST_U8(a) ((uint8_t)(a))
#define ST_U16(a) ((uint16_t)(a))
#define ST_U32(a) ((uint32_t)(a))
#define ST_U64(a) ((uint64_t)(a))
#define FD_I8(d) ((int8_t)(d))
#define FD_I16(d) ((int16_t)(d))
#define FD_I32(d) ((int32_t)(d))
#define FD_I64(d) ((int64_t)(d))
#define FD_U8(d) ((uint8_t)(d))
#define FD_U16(d) ((uint16_t)(d))
#define FD_U32(d) ((uint32_t)(d))
#define FD_U64(d) ((uint64_t)(d))

ORACLE_DEFINE(i8, int8_t, uint32_t, LD_U32, ST_I8, FD_I8, GT0, LT0, LT1, SIGN_SIGNED, ABS_I8);
ORACLE_DEFINE(i16, int16_t, uint32_t, LD_U32, ST_I16, FD_I16, GT0, LT0, LT1, SIGN_SIGNED, ABS_I8);
ORACLE_DEFINE(i32, int32_t, uint32_t, LD_U32, ST_I32, FD_I32, GT0, LT0, LT1, SIGN_SIGNED, ABS_I8);
ORACLE_DEFINE(i64, int64_t, uint64_t, LD_U64, ST_I64, FD_I64, GT0, LT0, LT1, SIGN_SIGNED, ABS_I64);
ORACLE_DEFINE(u8, uint8_t, uint32_t, LD_U32, ST_U8, FD_U8, GT0, LT0, LT1, SIGN_UNSIGNED, ABS_U32);
ORACLE_DEFINE(u16, uint16_t, uint32_t, LD_U32, ST_U16, FD_U16, GT0, LT0, LT1, SIGN_UNSIGNED, ABS_U32);
ORACLE_DEFINE(u32, uint32_t, uint32_t, LD_U32, ST_U32, FD_U32, GT0, LT0, LT1, SIGN_UNSIGNED, ABS_U32);
ORACLE_DEFINE(u64, uint64_t, uint64_t, LD_U64, ST_U64, FD_U64, GT0, LT0, LT1, SIGN_UNSIGNED, ABS_U64);

/* ---- double-carried twin of the f32 gradient (error analysis) ---- */
/* Every product and sum in double.  Rows are taken in panels of about 128 KB:
 * the panel's rows are widened to double once, its residuals are formed with
 * eight interleaved partial sums per dot product (float products are exact
 * in double, so the order only moves the last bits of a double sum), and the
 * accumulation into each chunk's gradient adds the rows in ascending order
 * for every element, features tiled so that the rows being updated stay in
 * cache -- the shape that makes 2^20 x 4096 x 256 a matter of seconds. */
static inline double dot_f64_8(const double* x, const double* m, int64_t n) {
    double p0 = 0, p1 = 0, p2 = 0, p3 = 0, p4 = 0, p5 = 0, p6 = 0, p7 = 0;
    int64_t f = 0;
    for (; f + 8 <= n; f += 8) {
        p0 += x[f + 0] * m[f + 0];
        p1 += x[f + 1] * m[f + 1];
        p2 += x[f + 2] * m[f + 2];
        p3 += x[f + 3] * m[f + 3];
        p4 += x[f + 4] * m[f + 4];
        p5 += x[f + 5] * m[f + 5];
        p6 += x[f + 6] * m[f + 6];
        p7 += x[f + 7] * m[f + 7];
    }
    double s = ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7));
    for (; f < n; ++f) s += x[f] * m[f];
    return s;
}

void oracle_glm_gradient_f32_acc64(const float* X, const float* M, const float* Y, double* grad,
                                   int64_t nf, int64_t nt, int64_t ntasks, int64_t nobs,
                                   double lambda, double alpha, int with_reg) {
    const int64_t K = nt * nf;
    if (K == 0) return;
    const int nth = oracle_get_threads();
    const int64_t panel = oracle_rows_per_group(nf * (int64_t)sizeof(double));
    double* Md = (double*)malloc((size_t)K * sizeof(double));
    for (int64_t task = 0; task < ntasks; ++task) {
        const float* Mt = M + task * K;
        for (int64_t k = 0; k < K; ++k) Md[k] = (double)Mt[k];
        double* g = grad + task * K;
        for (int64_t k = 0; k < K; ++k) g[k] = 0.0;
        const int64_t nchunks = ORACLE_MAX_CHUNKS;
        double* part = (double*)calloc((size_t)(nchunks * K), sizeof(double));
#pragma omp parallel for num_threads(nth) schedule(dynamic, 1)
        for (int64_t c = 0; c < nchunks; ++c) {
            double* acc = part + c * K;
            double* e = (double*)malloc((size_t)(panel * nt) * sizeof(double));
            double* xd = (double*)malloc((size_t)(panel * nf) * sizeof(double));
            const int64_t c0 = c * nobs / nchunks, c1 = (c + 1) * nobs / nchunks;
            for (int64_t o0 = c0; o0 < c1; o0 += panel) {
                const int64_t np = (o0 + panel < c1 ? o0 + panel : c1) - o0;
                for (int64_t p = 0; p < np; ++p) {
                    const float* x = X + ((o0 + p) * ntasks + task) * nf;
                    double* xr = xd + p * nf;
                    for (int64_t f = 0; f < nf; ++f) xr[f] = (double)x[f];
                }
                for (int64_t t = 0; t < nt; ++t)
                    for (int64_t p = 0; p < np; ++p)
                        e[p * nt + t] = dot_f64_8(xd + p * nf, Md + t * nf, nf) -
                                        (Y ? (double)Y[((o0 + p) * ntasks + task) * nt + t] : 0.0);
                for (int64_t f0 = 0; f0 < nf; f0 += ORACLE_FT) {
                    const int64_t f1 = f0 + ORACLE_FT < nf ? f0 + ORACLE_FT : nf;
                    for (int64_t t = 0; t < nt; ++t) {
                        double* row = acc + t * nf;
                        for (int64_t p = 0; p < np; ++p) {
                            const double et = e[p * nt + t];
                            const double* xr = xd + p * nf;
                            for (int64_t f = f0; f < f1; ++f) row[f] += et * xr[f];
                        }
                    }
                }
            }
            free(e);
            free(xd);
        }
        for (int64_t k = 0; k < K; ++k) {
            double s = 0.0;
            for (int64_t c = 0; c < nchunks; ++c) s += part[c * K + k];
            double v = 2.0 * s;
            if (with_reg && lambda > 0) {
                const double mv = (double)Mt[k];
                if (alpha > 0) v += lambda * alpha * (double)SIGN_SIGNED(mv);
                if (alpha < 1) v += 2.0 * lambda * (1.0 - alpha) * mv;
            }
            g[k] = v;
        }
        free(part);
    }
    free(Md);
}

/* ---- elastic-net proximal gradient (no counterpart in the reference) ---- */

/* SplitMix64 (Steele, Lea & Flood, OOPSLA 2014), top 53 bits to [-1, 1). */
static uint64_t splitmix64_next(uint64_t* state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void oracle_power_start(double* v0, int64_t n, uint64_t seed) {
    uint64_t state = seed;
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t r = splitmix64_next(&state) >> 11;
        v0[i] = 2.0 * ((double)r * (1.0 / 9007199254740992.0)) - 1.0;
    }
}

/* soft threshold S(z, t) = sign(z) * max(|z| - t, 0) */
static inline double soft_threshold(double z, double t) {
    const double a = fabs(z) - t;
    if (a <= 0.0) return 0.0;
    return z > 0.0 ? a : -a;
}

#define ORACLE_DEFINE_FIT(SFX, T)                                                            \
    void oracle_prox_step_##SFX(T* beta, const T* grad_smooth, int64_t n, double inv_L,     \
                                double l1) {                                                \
        const double thr = l1 * inv_L;                                                      \
        for (int64_t i = 0; i < n; ++i) {                                                   \
            const double z = (double)beta[i] - (double)grad_smooth[i] * inv_L;              \
            beta[i] = (T)soft_threshold(z, thr);                                            \
        }                                                                                   \
    }                                                                                       \
                                                                                            \
    void oracle_power_norm_##SFX(const T* X, const T* v0, int64_t nf, int64_t ntasks,       \
                                 int64_t nobs, int n_power, double* norm_out) {             \
        T* v = (T*)malloc((size_t)(nf * ntasks) * sizeof(T));                               \
        T* g = (T*)malloc((size_t)(nf * ntasks) * sizeof(T));                               \
        for (int64_t task = 0; task < ntasks; ++task) {                                     \
            double s = 0.0;                                                                 \
            for (int64_t f = 0; f < nf; ++f) s += (double)v0[task * nf + f] * (double)v0[task * nf + f]; \
            const double inv = s > 0.0 ? 1.0 / sqrt(s) : 0.0;                               \
            for (int64_t f = 0; f < nf; ++f) v[task * nf + f] = (T)((double)v0[task * nf + f] * inv); \
            norm_out[task] = 0.0;                                                           \
        }                                                                                   \
        for (int it = 0; it < n_power; ++it) {                                              \
            oracle_glm_gradient_##SFX(X, v, NULL, g, nf, 1, ntasks, nobs, 0.0, 0.0, 0);     \
            for (int64_t task = 0; task < ntasks; ++task) {                                 \
                double s = 0.0;                                                             \
                for (int64_t f = 0; f < nf; ++f) s += (double)g[task * nf + f] * (double)g[task * nf + f]; \
                const double nrm = sqrt(s);                                                 \
                const double inv = nrm > 0.0 ? 1.0 / nrm : 0.0;                             \
                for (int64_t f = 0; f < nf; ++f) v[task * nf + f] = (T)((double)g[task * nf + f] * inv); \
                norm_out[task] = nrm;                                                       \
            }                                                                               \
        }                                                                                   \
        free(v);                                                                            \
        free(g);                                                                            \
    }                                                                                       \
                                                                                            \
    void oracle_fit_##SFX(const T* X, const T* Y, T* beta, int64_t nf, int64_t nt,          \
                          int64_t ntasks, int64_t nobs, double lambda1, double lambda2,     \
                          const T* v0, int n_power, int n_iter, double* lipschitz_out) {    \
        const int64_t K = nf * nt;                                                          \
        double* nrm = (double*)malloc((size_t)ntasks * sizeof(double));                     \
        T* g = (T*)malloc((size_t)(K * ntasks) * sizeof(T));                                \
        oracle_power_norm_##SFX(X, v0, nf, ntasks, nobs, n_power, nrm);                     \
        for (int64_t task = 0; task < ntasks; ++task)                                       \
            lipschitz_out[task] = ORACLE_POWER_SAFETY * nrm[task] + 2.0 * lambda2;          \
        for (int64_t i = 0; i < K * ntasks; ++i) beta[i] = (T)0;                            \
        for (int it = 0; it < n_iter; ++it) {                                               \
            oracle_glm_gradient_##SFX(X, beta, Y, g, nf, nt, ntasks, nobs, lambda2, 0.0, 1); \
            for (int64_t task = 0; task < ntasks; ++task)                                   \
                oracle_prox_step_##SFX(beta + task * K, g + task * K, K,                    \
                                       1.0 / lipschitz_out[task], lambda1);                 \
        }                                                                                   \
        free(nrm);                                                                          \
        free(g);                                                                            \
    }                                                                                       \
    typedef int oracle_define_fit_##SFX##_done

ORACLE_DEFINE_FIT(f32, float);
ORACLE_DEFINE_FIT(f64, double);
