// Fused kernels of the device-resident QAT training step (SE-ResNet part).
// Every launcher takes device pointers only; scales and statistics stay on
// the device (no host round trip per conv, unlike the reference, which
// synchronises for every max-abs scale and BN statistic).
#pragma once
#include <vector>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace trba {
namespace qat {

constexpr float kBnEps = 1e-5f;

// Activation sources of the element-wise passes.
enum SrcKind {
    SRC_BN = 0,        // y = BN(x) from the forward trace
    SRC_FLOAT = 1,     // a stored fp32 tensor
    SRC_SE_RES_F = 2,  // z = y2 * gate[b,c] + res_f[i]          (downsample branch)
    SRC_SE_RES_Q = 3,  // z = y2 * gate[b,c] + q_in[i] * s_in    (identity branch)
    SRC_BN_EVAL = 4,   // y = BN(x) with the running statistics (inference)
};

struct Src {
    int kind;
    const float *x;       // SRC_BN: x; SRC_FLOAT / SRC_SE_*: y / y2
    const double *bn_acc; // SRC_BN: [2C] sum / sum of squares of x
    const float *run_mean, *run_var;  // SRC_BN_EVAL
    const float *gamma, *beta;
    const float *gate;    // SRC_SE_*: [B*C]
    const float *res_f;   // SRC_SE_RES_F
    const int8_t *res_q;  // SRC_SE_RES_Q
    const float *res_s;   // SRC_SE_RES_Q: device scalar
    int C, HW;
    i64 count;            // B*HW (BN statistics count)
};

// Pass 1 over a plane grid (one CTA per (b, c) plane): optional stores of y,
// the per-channel BN mean/var (channel CTAs of b == 0), the SE squeeze
// (per-plane mean of y, double sum / HW) and the running max|y| (atomicMax).
void act_stats(const Src &s, int B, float *y_out, float *mean_out, float *var_out, float *pool_out, float *vmax,
               cudaStream_t st);
// Pass 2: q = quantise(v) with s = max(vmax/127, 1e-12) (written to s_out);
// relu ? rint(min(max(v,0)/s, 127)) : rint(clamp(v/s, +-127)).
void act_quant(const Src &s, int B, const float *vmax, float *s_out, int8_t *q, bool relu, cudaStream_t st);

// SE excitation (src/qnet.rs:1211-1222): gate = sigmoid(fc2 relu(fc1 pool)).
void se_forward(const float *pool, const float *w1, const float *w2, int B, int C, int R, float *h1, float *gate,
                cudaStream_t st);

// Block-gradient entry and SE backward (src/qnet.rs:1684-1708, 1290-1296,
// 1298-1330) in one kernel: v = gv * s_out, s_dq = max(vmax/127, 1e-12),
// dq = rint(clamp(v/s_dq)), dz = q_out > 0 ? dq * s_dq : 0 (written), then
// the SE squeeze / excitation backward and dy2_full = dz*gate + dpooled/HW.
// vmax = max |gv * s_out| over the batch, accumulated by the producer of gv.
void se_backward(const float *gv, const float *s_out, const float *vmax, const int8_t *q_out, float *s_dq_out,
                 float *dz, const float *y2, const float *gate, const float *h1, const float *w1, const float *w2,
                 int B, int C, int HW, int R, float *dpre1, float *dpre2, float *dpooled, float *dy2_full,
                 cudaStream_t st);
void se_weight_grads(const float *dpre1, const float *dpre2, const float *h1, const float *pool, int B, int C, int R,
                     float *g_w1, float *g_w2, cudaStream_t st);

// Conv backward pieces (src/qnet.rs:937-1081).
void bn_bwd_sums(const float *dy, const float *x, const float *mean, const float *var, int B, int C, int HW,
                 double *acc, cudaStream_t st);
void bn_dx_max(const float *dy, const float *x, const float *mean, const float *var, const float *gamma,
               const double *acc, int B, int C, int HW, float *g_gamma, float *g_beta, float *vmax, cudaStream_t st);
// compat: A[o*ld + r] = qdx_flat[r*C + o] (transpose_i8 of the NCHW buffer
// viewed as [rows, C]); correct: A[o*ld + b*HW + p] = qdx[b, o, p].
void bn_dx_quant(const float *dy, const float *x, const float *mean, const float *var, const float *gamma,
                 const double *acc, int B, int C, int HW, const float *vmax, float *s_dx, int8_t *A, int ld,
                 bool compat, cudaStream_t st);
// g[i] += (float)acc[i] * (s_dx * s_in)
void grad_accum(const int32_t *acc, const float *s_dx, const float *s_in, i64 n, float *g, cudaStream_t st);
// Input gradient (gather over taps and output channels in the reference
// order) times w_s, then: mask_q ? (mask_q > 0 ? v : 0) : v, then + add.
// wT: (float) of the int8 weights at dgrad_weights_index; perm / cstart:
// the tap-class pixel order of dgrad_classes (device copies), or null for
// the natural order.  With gmax_out, atomically maxes max |gi * *gmax_scale|
// into *gmax_out (a non-negative f32, zeroed by the caller) — the
// re-quantisation scale of the block that consumes gi.
void dgrad(const float *dy, const float *wT, const float *w_s, int B, int Cin, int H, int W, int Cout, int kh, int kw,
           int sh, int sw, int ph, int pw, int Ho, int Wo, const int *perm, const int *cstart, int ncls,
           const int8_t *mask_q, const float *add, float *gi, cudaStream_t st, const float *gmax_scale = nullptr,
           float *gmax_out = nullptr);
// Floats of the input-gradient weight layout [Cin / 16 blocks][taps][Cout][16].
i64 dgrad_weights_size(int Cin, int Cout, int khw);
// Index in that layout of weight (oc, ci, tap).
__host__ __device__ inline i64 dgrad_weights_index(int oc, int ci, int tap, int Cout, int khw) {
    return (((i64)(ci >> 4) * khw + tap) * Cout + oc) * 16 + (ci & 15);
}
// Pixels of one image grouped by the set of taps valid for them (rows_only:
// by the valid kernel rows), classes in a fixed order: perm[H*W] image-local
// pixel indices, cstart[classes + 1]; both empty when there is one class.
void dgrad_classes(int H, int W, int kh, int kw, int sh, int sw, int ph, int pw, int Ho, int Wo, bool rows_only,
                   std::vector<int> &perm, std::vector<int> &cstart);
// Transposed im2col for the correct-mode weight gradient: colT[n*ld + r].
void im2col_t(const int8_t *in, int8_t *colT, int B, int C, int H, int W, int kh, int kw, int sh, int sw, int ph,
              int pw, int Ho, int Wo, int ld, cudaStream_t st);

// Stem pool input gradient (src/qnet.rs:1711-1729): gv *= s_pool, scatter
// through the 2x2 max of q1, mask by q1 > 0.
void pool_bwd_mask(const int8_t *q1, const float *gv, const float *s_pool, int B, int C, int H, int W, float *dy,
                   cudaStream_t st);
// Features (src/qnet.rs:1618-1622): feat[b,w,c] = sum_h (q*s) / H, and its
// backward fused with the output ReLU mask (src/qnet.rs:1642-1652).
void features(const int8_t *q, const float *s, int B, int C, int H, int W, float *feat, cudaStream_t st);
void features_bwd(const float *dfeat, const int8_t *q, const float *s, int B, int C, int H, int W, float *dy,
                  cudaStream_t st);
// dy = q > 0 ? g : 0 (the ReLU mask of a quantised activation).
void mask_by_q(const int8_t *q, const float *g, i64 n, float *dy, cudaStream_t st);

}  // namespace qat
}  // namespace trba
