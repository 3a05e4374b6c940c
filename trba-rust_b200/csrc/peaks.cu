// Measured ceiling of the arithmetic the exact input-gradient gather runs on:
// separately rounded f32 multiplies and adds, issued as packed f32x2 pairs.
#include "common.cuh"
#include "f32x2.cuh"
#include "trba_b200.h"

namespace trba {
namespace {

constexpr int kPeakChains = 8, kPeakIters = 4096, kPeakThreads = 256;

__device__ float g_peak_sink;

// Every thread runs kPeakChains chains with the instruction pair the gather
// uses (fma.rn.f32x2 with a run-time -0 addend, then add.rn.f32x2):
// acc[j] += acc[j-1] * w[j], all products of an iteration taken from the
// previous iteration's accumulators, so nothing is loop-invariant and the
// chains stay independent within an iteration.  No memory traffic.
__global__ void __launch_bounds__(kPeakThreads) f32_muladd_peak_kernel(float d0, float w0, float neg_zero) {
    const f32x2 z = pack2(neg_zero, neg_zero);
    f32x2 acc[kPeakChains], w[kPeakChains];
#pragma unroll
    for (int j = 0; j < kPeakChains; ++j) {
        acc[j] = pack2(d0 + (float)threadIdx.x, d0 - (float)(blockIdx.x + j));
        w[j] = pack2(w0 * (float)(j + 1), -w0 * (float)(j + 1));
    }
    for (int it = 0; it < kPeakIters; ++it) {
        f32x2 p[kPeakChains];
#pragma unroll
        for (int j = 0; j < kPeakChains; ++j) p[j] = prod2_rn(acc[(j + kPeakChains - 1) % kPeakChains], w[j], z);
#pragma unroll
        for (int j = 0; j < kPeakChains; ++j) acc[j] = add2_rn(acc[j], p[j]);
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < kPeakChains; ++j) {
        float lo, hi;
        unpack2(acc[j], lo, hi);
        s += lo + hi;
    }
    if (s == 1.2345f) g_peak_sink = s;  // keeps the chains live
}

}  // namespace
}  // namespace trba

using namespace trba;

extern "C" int trba_measure_f32_muladd_peak(double *tflops, void *stream) {
    if (!tflops) return -1;
    cudaStream_t st = as_stream(stream);
    const int blocks = sm_count() * 8;
    cudaEvent_t e0, e1;
    TRBA_CHECK(cudaEventCreate(&e0));
    TRBA_CHECK(cudaEventCreate(&e1));
    float best = 1e30f;
    for (int rep = 0; rep < 4; ++rep) {  // first launch warms up
        TRBA_CHECK(cudaEventRecord(e0, st));
        f32_muladd_peak_kernel<<<blocks, kPeakThreads, 0, st>>>(1e-3f, 1e-4f, -0.0f);
        TRBA_LAUNCH_CHECK();
        TRBA_CHECK(cudaEventRecord(e1, st));
        TRBA_CHECK(cudaEventSynchronize(e1));
        float ms = 0.0f;
        TRBA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        if (rep > 0 && ms < best) best = ms;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    // per chain step: 2 lanes x (1 multiply + 1 add)
    const double flops = (double)blocks * kPeakThreads * kPeakIters * kPeakChains * 4.0;
    *tflops = flops / (best * 1e-3) / 1e12;
    return 0;
}
