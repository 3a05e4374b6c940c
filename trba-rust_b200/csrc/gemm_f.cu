// fp32 and fp16 GEMMs of the drop-in ABI (src/backend.rs:26-27 of the
// reference's later snapshot).  Neither is on the QAT training path (the
// reference declares launch_gemm_fp16 but never calls it; launch_gemm_fp32 is
// used by its tests), so both are plain shared-memory tiled CUDA-core
// kernels, 64x64 tiles, 4x4 outputs per thread, fp32 accumulation.
#include <cuda_fp16.h>

#include "common.cuh"

namespace {

// C[M,N] = A[M,K] . B[K,N] (row-major, compact).
__global__ void gemm_f32_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                float *__restrict__ C, int M, int N, int K) {
    __shared__ float sa[16][65], sb[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int e = threadIdx.x; e < 64 * 16; e += 256) {
            const int r = e >> 4, k = e & 15;
            sa[k][r] = (m0 + r < M && k0 + k < K) ? A[(i64)(m0 + r) * K + k0 + k] : 0.f;
            const int kk = e >> 6, c = e & 63;
            sb[kk][c] = (k0 + kk < K && n0 + c < N) ? B[(i64)(k0 + kk) * N + n0 + c] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += sa[k][ty * 4 + i] * sb[k][tx * 4 + j];
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            const int r = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
            if (r < M && c < N) C[(i64)r * N + c] = acc[i][j];
        }
}

// C[M,N] = A[M,K] . Bt[N,K]^T, f16 operands with leading dimension align16(K).
__global__ void gemm_f16_kernel(const __half *__restrict__ A, const __half *__restrict__ B,
                                float *__restrict__ C, int M, int N, int K, int ld) {
    __shared__ float sa[16][65], sb[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int e = threadIdx.x; e < 64 * 16; e += 256) {
            const int r = e >> 4, k = e & 15;
            sa[k][r] = (m0 + r < M && k0 + k < K) ? __half2float(A[(i64)(m0 + r) * ld + k0 + k]) : 0.f;
            sb[k][r] = (n0 + r < N && k0 + k < K) ? __half2float(B[(i64)(n0 + r) * ld + k0 + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += sa[k][ty * 4 + i] * sb[k][tx * 4 + j];
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            const int r = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
            if (r < M && c < N) C[(i64)r * N + c] = acc[i][j];
        }
}

}  // namespace

using namespace trba;

extern "C" {

void launch_gemm_fp32(const float *a, const float *b, float *c, int m, int n, int k, void *s) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    // M tiles on grid.x (2^31-1 limit), N tiles on grid.y.
    dim3 grid((m + 63) / 64, (n + 63) / 64);
    TRBA_REQUIRE(grid.y <= 65535u, "launch_gemm_fp32: N too large");
    gemm_f32_kernel<<<grid, 256, 0, as_stream(s)>>>(a, b, c, m, n, k);
    TRBA_LAUNCH_CHECK();
}

void launch_gemm_fp16(const void *a, const void *b, float *c, int m, int n, int k, void *s) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    dim3 grid((m + 63) / 64, (n + 63) / 64);
    TRBA_REQUIRE(grid.y <= 65535u, "launch_gemm_fp16: N too large");
    gemm_f16_kernel<<<grid, 256, 0, as_stream(s)>>>((const __half *)a, (const __half *)b, c, m, n, k,
                                                    (k + 15) & ~15);
    TRBA_LAUNCH_CHECK();
}

}  // extern "C"
