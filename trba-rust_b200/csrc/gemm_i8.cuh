// Host-side entry points of the tcgen05 int8 GEMM (gemm_i8.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace trba {

// 2-D int8 tensor map over rows x k (leading dimension ld bytes), boxes of
// 128 bytes of K by box_rows rows, 128-byte swizzle, zero fill outside.
bool make_tmap_i8(CUtensorMap *m, const void *ptr, int rows, int k, int ld, int box_rows);
int pick_bn(int N);
// C[M,N] s32 = A . Bt^T (compact C).  False if a tensor map cannot describe
// the operands (caller falls back to gemm_i8_simt).
bool gemm_i8_tc(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld, cudaStream_t st);
// C (pre-zeroed) += A . Bt^T with K split `splits` ways, integer atomics.
bool gemm_i8_splitk_atomic(const int8_t *A, int lda, const int8_t *B, int ldb, int32_t *C, int M, int N, int K,
                           int splits, cudaStream_t st);
// Conv forward: x[b, n, p] = (float)acc[r = b*HW + p, n] * (s_in * w_s), and
// bn_acc[n] += sum x, bn_acc[N + n] += sum x^2 (f64).  N <= 512.  w_s is a
// device scalar, or (per_channel) one scale per output channel n.
bool gemm_i8_conv_f32(const int8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, float *x,
                      const float *s_in, const float *w_s, bool per_channel, double *bn_acc, int HW,
                      cudaStream_t st);
// Fused epilogues on row-major outputs [M, N]: the conv inference requant
// (int8) and per-channel dequantisation (f32, optional bias and ReLU).
bool gemm_i8_requant(const int8_t *A, const int8_t *B, int8_t *out, const float *bias, int M, int N, int K, int ld,
                     float div, float mul, cudaStream_t st);
bool gemm_i8_dequant(const int8_t *A, const int8_t *B, float *out, const float *w_scale, float a_scale,
                     const float *bias, int relu, int M, int N, int K, int ld, cudaStream_t st);
// Implicit-GEMM conv forward: the GEMM's A rows gathered from NHWC int8
// activations x [B, H, W, Cin] (Cin a power of two >= 16, x 16-byte aligned)
// in K order (ky, kx, ci); Wh = the int8 weights in that K order,
// [N, kh*kw*Cin] with leading dimension ldw (a multiple of 16).  Row r of the
// result is output pixel (b, oy, ox), as with im2col.
struct ConvGeo {
    const int8_t *x;
    int B, H, W, Cin, kh, kw, sh, sw, ph, pw, Ho, Wo;
};
bool conv_implicit_ok(const ConvGeo &g);
// The conv forward epilogue of gemm_i8_conv_f32 over the gathered operand.
bool gemm_i8_conv_implicit_f32(const ConvGeo &g, const int8_t *Wh, int ldw, int N, float *x, const float *s_in,
                               const float *w_s, bool per_channel, double *bn_acc, cudaStream_t st);
// s32 accumulators, compact C [B*Ho*Wo, N].
bool gemm_i8_conv_implicit_s32(const ConvGeo &g, const int8_t *Wh, int ldw, int N, int32_t *C, cudaStream_t st);
int splitk_for(int M, int N, int K);
void gemm_i8_simt(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld, cudaStream_t st);

}  // namespace trba
