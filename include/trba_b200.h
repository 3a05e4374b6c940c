/*
 * trba_b200.h — entry points of libtrba_b200.so that have no counterpart in
 * the reference's ABI: diagnostics of the tensor-core kernels.  (The fused
 * training-step API lives in trba_qat.h.)
 */
#ifndef TRBA_B200_H
#define TRBA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* launch_gemm_int8 routed through the CUDA-core (dp4a) kernel that serves
 * operands a tensor map cannot describe (base not 16-byte aligned). */
void trba_gemm_int8_simt(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k,
                         void *stream);

/* Split-K variant of launch_gemm_int8 for long K: C (zeroed by the caller)
 * += A . Bt^T, K split `splits` ways (0 = automatic), partial tiles combined
 * with integer atomics (exact, order-independent). */
void trba_gemm_int8_splitk(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k, int splits,
                           void *stream);

/* C[M,N] = A[M,K] . B[K,N] (fp32, row-major, compact C; the contract of
 * launch_gemm_fp32) with f64 accumulation and split-K, allocating nothing:
 * its split-K scratch is a static 8 MiB device array.  For callers that may
 * not allocate device memory (plugins whose host owns every allocation,
 * loops where cudaMalloc would synchronise the device).  At most 131072
 * outputs (M*N) per call, larger calls return -1 with an error.  The first
 * call on a device looks up the array's address: make it before any stream
 * capture.  All calls share the array, so calls overlapping on the GPU race.
 * No counterpart in the reference's ABI.  Returns 0 or an error code. */
int trba_sgemm_exact_noalloc(const float *a, const float *b, float *c, int m, int n, int k, void *stream);

/* Number of kernels this library has launched so far (every launch site
 * counts itself), for reporting launches per step. */
/* Measured ceiling (no counterpart in the reference) of separately rounded
 * f32 multiply + add pairs issued as packed f32x2 instructions — the
 * arithmetic of the exact input-gradient gather: a kernel of independent
 * chains on every SM, timed with CUDA events; *tflops counts the multiply
 * and the add as one flop each.  Synchronises the stream. */
int trba_measure_f32_muladd_peak(double *tflops, void *stream);
/* GEMM with the conv inference epilogue fused (no counterpart in the
 * reference; equal to launch_gemm_int8 followed by launch_conv_epilogue(acc,
 * bias, out, n, acc_div, out_mul, m, n, 1, 1)): out int8 [m, n] =
 * rint(clamp(max(acc/acc_div + bias[n], 0) * out_mul, +-127)).  Operands as
 * launch_gemm_int8. */
void trba_gemm_int8_requant(const int8_t *a, const int8_t *b, const float *bias, int8_t *out, int m, int n, int k,
                            float acc_div, float out_mul, void *stream);
/* GEMM with per-output-channel dequantisation fused (no counterpart in the
 * reference): out f32 [m, n] = act((float)acc * (a_scale * w_scale[n])
 * [+ bias[n]]), act = ReLU when relu != 0.  bias may be NULL. */
void trba_gemm_int8_dequant_f32(const int8_t *a, const int8_t *b, const float *w_scale, float a_scale,
                                const float *bias, int relu, float *out, int m, int n, int k, void *stream);
long long trba_launch_count(void);
/* Large int8 GEMMs (unsplit, N a multiple of 256, at least one wave of
 * 256 x 256 tiles) run on CTA pairs (tcgen05 cta_group::2); enable = 0 routes
 * them to the single-CTA kernel instead (same results bit for bit; used by
 * the tests to compare the two).  Returns the previous setting.  No
 * counterpart in the reference. */
int trba_gemm_pair_enable(int enable);

/* launch_conv_backward_grad_input_i8 (reference backend.rs:51, the later
 * snapshot's cuda/kernels.cu:913-957) on the tensor cores: an implicit GEMM
 * per stride-phase class of input pixels (tcgen05 kind::f16, the fp32
 * output gradient as three bf16 terms whose sum is exact, the int8 weights
 * exact in bf16, fp32 accumulation).  Stride-1 convs (Cout % 16 == 0,
 * padding below the kernel size) use the halo tiling instead: dy on a
 * zero-padded grid, one shared-memory halo per tile serving every tap as a
 * shifted window.  Same arguments and result as the reference launcher up
 * to the order of the fp32 additions (relative differences around 1e-6 of
 * the gradient's scale).  Needs Cout a power of two >= 8, at most 4 stride
 * phases and 16 taps per phase.  Keeps a grow-only per-device buffer for
 * the bf16 weight image and the dy planes.  Returns 0, -1 for an
 * unsupported conv, or a CUDA error code. */
int trba_conv_grad_input_i8_tc(const float *grad_out, const int8_t *weight_q, int w_ld, float w_scale,
                               float *grad_input, int b, int cin, int h, int w, int cout, int kh, int kw,
                               int sh, int sw, int ph, int pw, int ho, int wo, void *stream);

/* Check of the division in the fused requant epilogue of
 * trba_gemm_int8_requant (no counterpart in the reference): for 2^-90 <=
 * |div| <= 2^90 the epilogue divides each s32 accumulator by div with an
 * FMA-based correctly rounded division against a host-computed reciprocal
 * (outside that range it uses the IEEE division).  Runs all 2^32 s32
 * accumulator values through both divisions on the device and returns how
 * many results differ in any bit (0 expected), or -1 when div is outside the
 * FMA path's range.  Synchronises the stream. */
long long trba_requant_division_check(float div, void *stream);

/* launch_im2col_pad followed by launch_gemm_int8 (reference backend.rs,
 * cuda/kernels.cu:476-541 and :227-250: the QAT conv forward's GEMM,
 * src/qnet.rs:338-458) as one implicit GEMM on the tensor cores (tcgen05
 * kind::i8): the receptive field of each output pixel is gathered into the
 * GEMM's shared-memory stages straight from the activations, so the im2col
 * matrix is never written.  acc = s32 [b*ho*wo, cout] compact, bit for bit
 * what im2col + GEMM give (integer sums do not depend on the K order).
 * input: int8 NCHW [b, cin, h, w]; weight_q: [cout, w_ld] in the reference's
 * (ci, ky, kx) K order, w_ld >= cin*kh*kw.  Needs cin a power of two in
 * [16, 1024].  Keeps a grow-only per-device buffer for the channel-innermost
 * copy of the input and the re-ordered weights.  Returns 0, -1 for an
 * unsupported conv, or a CUDA error code. */
int trba_conv_gemm_int8_implicit(const int8_t *input, const int8_t *weight_q, int w_ld, int32_t *acc, int b,
                                 int cin, int h, int w, int cout, int kh, int kw, int sh, int sw, int ph, int pw,
                                 int ho, int wo, void *stream);

/* Self-test of the bounded waits of the tensor-core kernels (no
 * counterpart in the reference): runs one small tensor-core input-gradient
 * launch of each tiling (class and halo) whose weight copies are
 * deliberately never issued, so its pipeline waits give up after limit_ns
 * instead of hanging; each kernel releases its tensor memory and raises the
 * device error word.  Synchronises the stream; returns 1 when both launches
 * gave up as designed (the word is cleared after each), or the other
 * launch's error word / a negative value / a CUDA error code. */
int trba_tc_wait_selftest(unsigned long long limit_ns, void *stream);

/* Tiling of the tensor-core input gradient for plans made after the call
 * (process wide; no counterpart in the reference, for tests and tuning):
 * mb < 0 keeps every conv on the class tiling, mb == 0 (the default) lets a
 * cost model pick the halo tile of stride-1 convs, mb = 1 .. 4 forces
 * 128 * mb positions per halo tile, and kc = 16, 32 or 64 forces the output
 * channels per halo stage (0: chosen). */
void trba_tc_dgrad_tiling(int mb, int kc);

/* Host-side plan of the tensor-core input gradient of a conv at batch b (no
 * counterpart in the reference; no GPU work): fills up to n_out fields of
 * out (tiling, tile counts, halo geometry, scratch and shared-memory sizes,
 * per-tap offsets; the order is documented at the definition) and returns
 * how many the plan has, or -1 when the conv is not served. */
int trba_tc_dgrad_plan(int b, int cin, int h, int w, int cout, int kh, int kw, int sh, int sw, int ph, int pw,
                       int ho, int wo, long long *out, int n_out);

/* Device error word of the tensor-core kernels: 1 when a bounded mbarrier
 * wait gave up.  Synchronises the device; clears the word if clear != 0. */
int trba_tc_error_poll(int clear);

#ifdef __cplusplus
}
#endif
#endif
