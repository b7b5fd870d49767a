// f64_mma_probe.cu -- the double-precision tensor-core MMA shapes on sm_100a.
//
// The tiled float64 gradient (gpu_algos_b200/csrc/glm_tiles.cu) feeds
// mma.sync m16n8k16 f64 from shared memory with a fixed assignment of matrix
// elements to lanes.  This probe checks that assignment for every f64 shape
// (m8n8k4, m16n8k4, m16n8k8, m16n8k16) against a host product, one warp, all
// indexes inside 256-element buffers, and measures each shape's issue
// throughput (operands in registers, independent accumulators, two CTAs of 8
// warps per SM): the FP64 tensor pipe's peak that the tiled kernel is held
// against.  Prints one "layout" line per shape ("ok" or "MISMATCH") and one
// "tput" line per (shape, accumulator count).
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <cmath>
#include <cuda_runtime.h>

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e_), __LINE__); return 1; } } while (0)

// ---- one MMA per shape, fragments loaded and stored by these layouts ----
// g = lane>>2, t = lane&3
// m8n8k4 : a(g,t)  b(t,g)  c(g, 2t+i)
// m16n8k4: a_i(g+8i, t)             b(t,g)             c_i(g+8(i>>1), 2t+(i&1))
// m16n8k8: a_i(g+8(i&1), t+4(i>>1)) b_i(t+4i, g)       c as above
// m16n8k16:a_i(g+8(i&1), t+4(i>>1)) b_i(t+4i, g)       c as above
template <int SH>
__global__ void layout_kernel(const double* A, const double* B, double* D) {
    const int lane = threadIdx.x, g = lane >> 2, t = lane & 3;
    if (SH == 0) {  // m8n8k4: A 8x4, B 4x8
        double a = A[g * 4 + t], b = B[t * 8 + g], d0 = 0, d1 = 0;
        asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                     : "+d"(d0), "+d"(d1) : "d"(a), "d"(b));
        D[g * 8 + 2 * t] = d0;
        D[g * 8 + 2 * t + 1] = d1;
        return;
    }
    double c[4] = {0, 0, 0, 0};
    if (SH == 1) {  // m16n8k4: A 16x4, B 4x8
        double a0 = A[g * 4 + t], a1 = A[(g + 8) * 4 + t], b0 = B[t * 8 + g];
        asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                     : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3]) : "d"(a0), "d"(a1), "d"(b0));
    } else if (SH == 2) {  // m16n8k8: A 16x8, B 8x8
        double a[4], b[2];
        for (int i = 0; i < 4; ++i) a[i] = A[(g + 8 * (i & 1)) * 8 + t + 4 * (i >> 1)];
        for (int i = 0; i < 2; ++i) b[i] = B[(t + 4 * i) * 8 + g];
        asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                     : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
    } else {  // m16n8k16: A 16x16, B 16x8
        double a[8], b[4];
        for (int i = 0; i < 8; ++i) a[i] = A[(g + 8 * (i & 1)) * 16 + t + 4 * (i >> 1)];
        for (int i = 0; i < 4; ++i) b[i] = B[(t + 4 * i) * 8 + g];
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, {%12,%13,%14,%15}, {%0,%1,%2,%3};"
                     : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                     : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]),
                       "d"(b[0]), "d"(b[1]), "d"(b[2]), "d"(b[3]));
    }
    for (int i = 0; i < 4; ++i) D[(g + 8 * (i >> 1)) * 8 + 2 * t + (i & 1)] = c[i];
}

// ---- throughput: NACC independent accumulators per warp ----
template <int SH, int NACC>
__global__ void __launch_bounds__(256) tput_kernel(double* out, int iters, double seed) {
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    double a[8], b[4];
    for (int i = 0; i < 8; ++i) a[i] = seed * (1 + i + (threadIdx.x & 7));
    for (int i = 0; i < 4; ++i) b[i] = seed * (2 + i + (threadIdx.x & 3));
    double c[NACC][4];
    for (int j = 0; j < NACC; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < NACC; ++j) {
            if (SH == 0) {
                asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                             : "+d"(c[j][0]), "+d"(c[j][1]) : "d"(a[j & 7]), "d"(b[j & 3]));
            } else if (SH == 1) {
                asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                             : "+d"(c[j][0]), "+d"(c[j][1]), "+d"(c[j][2]), "+d"(c[j][3])
                             : "d"(a[0]), "d"(a[1]), "d"(b[j & 3]));
            } else if (SH == 2) {
                asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                             : "+d"(c[j][0]), "+d"(c[j][1]), "+d"(c[j][2]), "+d"(c[j][3])
                             : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
            } else {
                asm volatile("mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, {%12,%13,%14,%15}, {%0,%1,%2,%3};"
                             : "+d"(c[j][0]), "+d"(c[j][1]), "+d"(c[j][2]), "+d"(c[j][3])
                             : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]),
                               "d"(b[0]), "d"(b[1]), "d"(b[2]), "d"(b[3]));
            }
        }
    }
    double s = 0;
    for (int j = 0; j < NACC; ++j) s += c[j][0] + c[j][1] + c[j][2] + c[j][3];
    out[gt] = s;  // out holds gridDim.x * blockDim.x doubles
}

static const int kM[4] = {8, 16, 16, 16}, kN[4] = {8, 8, 8, 8}, kK[4] = {4, 4, 8, 16};
static const char* kName[4] = {"m8n8k4", "m16n8k4", "m16n8k8", "m16n8k16"};

template <int SH>
int check_layout() {
    const int M = kM[SH], N = kN[SH], K = kK[SH];
    std::vector<double> A(M * K), B(K * N), D(M * N), R(M * N, 0.0);
    for (int i = 0; i < M * K; ++i) A[i] = 1 + i % 7 + 0.001 * i;
    for (int i = 0; i < K * N; ++i) B[i] = 1 + i % 5 + 0.01 * i;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n)
            for (int k = 0; k < K; ++k) R[m * N + n] += A[m * K + k] * B[k * N + n];
    double *dA, *dB, *dD;
    CK(cudaMalloc(&dA, 256 * 8)); CK(cudaMalloc(&dB, 256 * 8)); CK(cudaMalloc(&dD, 256 * 8));
    CK(cudaMemset(dD, 0, 256 * 8));
    CK(cudaMemcpy(dA, A.data(), M * K * 8, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dB, B.data(), K * N * 8, cudaMemcpyHostToDevice));
    layout_kernel<SH><<<1, 32>>>(dA, dB, dD);
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(D.data(), dD, M * N * 8, cudaMemcpyDeviceToHost));
    int bad = 0;
    for (int i = 0; i < M * N; ++i)
        if (std::fabs(D[i] - R[i]) > 1e-9 * std::fabs(R[i])) ++bad;
    printf("layout %-9s: %s (%d of %d wrong)\n", kName[SH], bad ? "MISMATCH" : "ok", bad, M * N);
    cudaFree(dA); cudaFree(dB); cudaFree(dD);
    return 0;
}

template <int SH, int NACC>
int tput(int sms) {
    const int blocks = sms * 2, threads = 256, iters = 4096;
    double* out;
    CK(cudaMalloc(&out, size_t(blocks) * threads * 8));
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0)); CK(cudaEventCreate(&e1));
    tput_kernel<SH, NACC><<<blocks, threads>>>(out, 64, 1e-3);
    CK(cudaDeviceSynchronize());
    CK(cudaEventRecord(e0));
    tput_kernel<SH, NACC><<<blocks, threads>>>(out, iters, 1e-3);
    CK(cudaEventRecord(e1));
    CK(cudaEventSynchronize(e1));
    float ms;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    const double fma = double(kM[SH]) * kN[SH] * kK[SH];
    const double flops = 2.0 * fma * NACC * iters * (double(blocks) * threads / 32);
    printf("tput %-9s nacc=%d: %.3f ms  %.2f TFLOP/s\n", kName[SH], NACC, ms, flops / ms / 1e9);
    cudaFree(out);
    return 0;
}

int main() {
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
    if (check_layout<0>() || check_layout<1>() || check_layout<2>() || check_layout<3>()) return 1;
    if (tput<0, 4>(sms) || tput<0, 8>(sms) || tput<1, 4>(sms) || tput<1, 8>(sms) || tput<2, 2>(sms) ||
        tput<2, 4>(sms) || tput<3, 1>(sms) || tput<3, 2>(sms) || tput<3, 4>(sms))
        return 1;
    return 0;
}
