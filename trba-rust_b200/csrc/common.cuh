// Shared helpers of libtrba_b200: error handling, launch geometry, numerics.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

typedef long long i64;

namespace trba {

// Error policy.  The reference aborts on any CUDA error (cuda/kernels.cu:37-50);
// that stays the default.  With abort disabled the first error is kept in a
// sticky word until trba_clear_error().
void report_error(const char *file, int line, const char *what, int code);
bool abort_on_error();

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Streaming multiprocessors of the current device (148 on B200).
int sm_count();

// Grid for a grid-stride loop: enough CTAs to cover n items, capped at a
// whole number of waves (8 resident 256-thread CTAs per SM).
inline int grid_for(i64 n, int threads = 256) {
    i64 want = (n + threads - 1) / threads;
    i64 cap = (i64)sm_count() * 8;
    if (want < 1) want = 1;
    return (int)(want < cap ? want : cap);
}

}  // namespace trba

#define TRBA_CHECK(call)                                                      \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess) trba::report_error(__FILE__, __LINE__, cudaGetErrorString(e_), (int)e_); \
    } while (0)

// Every kernel launch of the library goes through this check, which also
// counts it (trba_launch_count()).
namespace trba {
void count_launch();
void count_launches(long long n);  // kernels replayed inside a CUDA graph
long long launches_so_far();
}
#define TRBA_LAUNCH_CHECK()          \
    do {                             \
        trba::count_launch();        \
        TRBA_CHECK(cudaGetLastError()); \
    } while (0)

// Shape contract violations (the reference's REQUIRE_SHAPE, cuda/kernels.cu
// of the later snapshot, lines 89-96): same policy as CUDA errors.
#define TRBA_REQUIRE(cond, msg)                                               \
    do {                                                                      \
        if (!(cond)) { trba::report_error(__FILE__, __LINE__, msg, -1); return; } \
    } while (0)

#define TRBA_REQUIRE_RET(cond, msg, ret)                                      \
    do {                                                                      \
        if (!(cond)) { trba::report_error(__FILE__, __LINE__, msg, -1); return ret; } \
    } while (0)

// Grid-stride loop over [0, n).
#define GRID_LOOP(i, n)                                                       \
    for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < (n);         \
         i += (i64)gridDim.x * blockDim.x)

// Device numerics written with explicit IEEE round-to-nearest intrinsics so
// that no multiply-add is contracted: results then match the reference CPU
// backend bit for bit wherever it evaluates the same expression in float.
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ int rint_even(float v) { return __float2int_rn(v); }

// Transcendentals of the training step, evaluated in f64 and rounded once to
// f32 (correctly rounded except in vanishingly rare ties).  The CPU oracle
// evaluates the same way, so both sides produce identical f32 results; the
// reference's f32 libm calls differ from these by at most an ulp.
__device__ __forceinline__ float cr_expf(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float cr_tanhf(float x) { return (float)tanh((double)x); }
__device__ __forceinline__ float cr_logf(float x) { return (float)log((double)x); }
__device__ __forceinline__ float cr_sigmoid(float x) { return fdiv(1.0f, fadd(1.0f, cr_expf(-x))); }
