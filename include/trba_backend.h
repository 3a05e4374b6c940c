/*
 * trba_backend.h — the drop-in C ABI of the TRBA INT8-QAT backend, built for
 * NVIDIA B200 (sm_100a) by libtrba_b200.so.
 *
 * Every declaration below replaces, with the same name, C types and argument
 * meaning, one entry of the `extern "C"` block that trba-rust binds in
 * src/backend.rs (later snapshot: src/backend.rs:14-143; checked-out tree:
 * src/backend.rs:14-83) or src/gpu_memory.rs:13-20.  The line cited beside
 * each entry is that binding.  Rust `i32` = int, `i64` = long long,
 * `usize` = size_t, `*mut c_void` stream = cudaStream_t (NULL = legacy
 * default stream).
 *
 * Contract (unchanged from the reference):
 *   - every pointer is a DEVICE pointer owned by the caller, except
 *     maxpool2x2_backward_host (host pointers);
 *   - int8 GEMM operands are row-major [align16(rows), align16(K)] and are
 *     read only for k < K and rows below M / N (tails need not be zero here);
 *     C is compact [M, N] int32;
 *   - launchers return silently on non-positive sizes;
 *   - work is enqueued on `stream`; results are valid after cuda_sync(stream).
 *
 * Errors: as in the reference, a CUDA error or an invalid shape prints
 * "[CUDA FATAL] ..." and aborts the process.  trba_set_abort_on_error(0)
 * switches to a sticky error word instead (read with trba_last_error()),
 * which is what the test-suite uses.
 */
#ifndef TRBA_BACKEND_H
#define TRBA_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------- runtime ----- */
void cuda_malloc(void **ptr, size_t size);                                   /* backend.rs:15 */
void cuda_free(void *ptr);                                                   /* backend.rs:16 */
void cuda_memcpy_h2d(void *dst, const void *src, size_t size, void *stream); /* backend.rs:17 */
void cuda_memcpy_dtod(void *dst, const void *src, size_t size, void *stream);/* backend.rs:18 */
void cuda_memcpy_d2h(void *dst, const void *src, size_t size, void *stream); /* backend.rs:19 */
void cuda_sync(void *stream);                                                /* backend.rs:20 */
void cuda_stream_create(void **stream);                                      /* backend.rs:21 */
void cuda_stream_destroy(void *stream);                                      /* backend.rs:22 */
void cuda_get_memory_info(size_t *free_mem, size_t *total_mem);              /* backend.rs:23 */

/* ------------------------------------------------------------ GEMMs ----- */
/* C[M,N] s32 = A[M,K] . Bt[N,K]^T on tcgen05 kind::i8 tensor cores.  backend.rs:25 */
void launch_gemm_int8(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k,
                      void *stream);
/* C[M,N] f32 = A[M,K] f16 . Bt[N,K]^T f16, same padding contract.  backend.rs:26 */
void launch_gemm_fp16(const void *a, const void *b, float *c, int m, int n, int k, void *stream);
/* C[M,N] = A[M,K] . B[K,N], fp32, compact.  backend.rs:27 */
void launch_gemm_fp32(const float *a, const float *b, float *c, int m, int n, int k, void *stream);

/* ------------------------------------------------------ conv helpers ---- */
/* int8 im2col into [align16(B*Ho*Wo), col_ld], K order (c,kh,kw), zero tails.  backend.rs:28 */
void launch_im2col_pad(const int8_t *input, int8_t *col, int batch, int c, int h, int w, int kh,
                       int kw, int sh, int sw, int ph, int pw, int ho, int wo, int col_ld,
                       void *stream);
/* fp32 compact im2col.  backend.rs:31 */
void launch_im2col_gpu(const int8_t *input, float *col, int batch, int c, int h, int w, int kh,
                       int kw, int sh, int sw, int ph, int pw, int ho, int wo, void *stream);
/* int8 NCHW = rint(clamp(max(acc/acc_div + bias, 0) * out_mul)).  backend.rs:34 */
void launch_conv_epilogue(const int32_t *acc, const float *bias, int8_t *out, int acc_ld,
                          float acc_div, float out_mul, int b, int c, int ho, int wo, void *stream);
/* fp32 weight gradient by direct sum (diagnostic path).  backend.rs:37 */
void launch_conv_backward_grad_weight(const int8_t *input, const float *grad_out, float *grad_w,
                                      int b, int cin, int h, int w, int cout, int kh, int kw,
                                      int sh, int sw, int ph, int pw, int ho, int wo, void *stream);
/* per-channel sum of grad_out.  backend.rs:41 */
void launch_conv_backward_grad_bias(const float *grad_out, float *grad_bias, int b, int cout,
                                    int ho, int wo, void *stream);
/* input gradient, fp32 weights [Cout, Cin*kh*kw].  backend.rs:43 */
void launch_conv_backward_grad_input(const float *grad_out, const float *weight, float *grad_input,
                                     int b, int cin, int h, int w, int cout, int kh, int kw, int sh,
                                     int sw, int ph, int pw, int ho, int wo, void *stream);
/* input gradient, int8 weights with leading dimension w_ld, times w_scale.  backend.rs:51 */
void launch_conv_backward_grad_input_i8(const float *grad_out, const int8_t *weight_q, int w_ld,
                                        float w_scale, float *grad_input, int b, int cin, int h,
                                        int w, int cout, int kh, int kw, int sh, int sw, int ph,
                                        int pw, int ho, int wo, void *stream);

/* ----------------------------------------------------------- maxpool ---- */
void maxpool2x2_backward_host(const float *grad_output, const uint64_t *max_indices,
                              float *grad_input, uint64_t output_size,
                              uint64_t input_size);                          /* backend.rs:56 */
void launch_maxpool2x2_backward(const float *grad_output, const int64_t *max_indices,
                                float *grad_input, long long output_size, long long input_size,
                                void *stream);                               /* backend.rs:58 */
void launch_maxpool2x2_forward_i8(const int8_t *x, int8_t *y, int b, int c, int h, int w,
                                  void *stream);                             /* backend.rs:105 */
void launch_maxpool2x2_backward_i8(const int8_t *x, const float *dy, float *dx, int b, int c,
                                   int h, int w, void *stream);              /* backend.rs:109 */

/* ------------------------------------------- conv optimiser state ------- */
/* g += acc * scale.  backend.rs:63 */
void launch_grad_accum_i32(const int32_t *acc, float *g, float scale, long long n, void *stream);
/* *out += sum(x^2) in f64.  backend.rs:68 */
void launch_sum_sq_add_f32(const float *x, double *out, long long n, void *stream);
/* momentum-free Muon step on one matrix.  backend.rs:91 */
void launch_muon_step_f32(float *p, const float *g, const double *gsq, long long n, double lr,
                          double wd, double clip, double min_dim, double max_dim, double cap,
                          long long autoscale, void *stream);
/* Adam with f64 intermediates.  backend.rs:94 */
void launch_adam_f32(float *p, const float *g, float *m, float *v, long long n, double lr,
                     double wd, double clip, double b1, double b2, double eps, double bc1,
                     double bc2, void *stream);
/* *out = max|x|.  backend.rs:98 */
void launch_max_abs_f32(const float *x, float *out, long long n, void *stream);
/* per-tensor weight fake-quant into the padded GEMM operand.  backend.rs:101 */
void launch_quantize_pad_i8(const float *w, const float *max_abs, float *w_s_out, int8_t *w_q_pad,
                            long long rows, long long col, long long kp, void *stream);

/* ------------------------------------------------------- BiLSTM fp32 ---- */
void launch_lstm_fwd_step(const float *x, const float *w_ih, const float *b_ih, const float *w_hh,
                          const float *b_hh, float *gates, float *c_out, float *h_out, long long b,
                          long long t, long long d, long long h, long long slot, long long rev,
                          void *stream);                                     /* backend.rs:74 */
void launch_lstm_bwd_cell(const float *dh_out, const float *gates, const float *ctrace,
                          const float *dh_next, const float *dc_next, float *dgates,
                          float *dc_next_out, long long b, long long h, long long slot,
                          void *stream);                                     /* backend.rs:78 */
void launch_lstm_bwd_rec(const float *dgates, const float *w_ih, const float *w_hh, float *dx,
                         float *dh_next, long long b, long long t, long long d, long long h,
                         long long slot, long long rev, void *stream);       /* backend.rs:82 */
void launch_lstm_wgrad_ih(const float *dgates, const float *x, float *g_w, long long b,
                          long long t, long long d, long long h, long long rev,
                          long long accumulate, void *stream);               /* backend.rs:85 */
void launch_lstm_wgrad_hh(const float *dgates, const float *htrace, float *g_w, long long b,
                          long long t, long long h, long long accumulate,
                          void *stream);                                     /* backend.rs:87 */
void launch_lstm_bgrad(const float *dgates, float *g_b_ih, float *g_b_hh, long long b, long long t,
                       long long h, long long accumulate, void *stream);     /* backend.rs:89 */

/* --------------------------------------------------------- utilities ---- */
void cuda_float_to_half(const float *src, void *dst, long long n, void *stream); /* backend.rs:111 */
void cuda_scale_vector(float *data, float scale, long long n, void *stream);     /* backend.rs:112 */
void cuda_transpose_f32(const float *src, float *dst, int rows, int cols, void *stream); /* :113 */

/* -------------------------------------------- BN / quantisation / SE ---- */
void launch_bn_stats(const float *x, int b, int c, int hw, float *mean, float *var,
                     void *stream);                                          /* backend.rs:115 */
void launch_bn_apply(const float *x, const float *mean, const float *var, const float *gamma,
                     const float *beta, float eps, float *y, int c, int hw, long long n,
                     void *stream);                                          /* backend.rs:116 */
void launch_bn_bwd_sums(const float *dy, const float *x, const float *mean, const float *var,
                        float eps, int c, int hw, long long n, float *sum_dy, float *sum_dy_xhat,
                        void *stream);                                       /* backend.rs:117 */
void launch_bn_bwd_dx(const float *dy, const float *x, const float *mean, const float *var,
                      const float *gamma, const float *sum_dy, const float *sum_dy_xhat, float eps,
                      int c, int hw, long long n, long long count, float *dx,
                      void *stream);                                         /* backend.rs:118 */
void launch_reduce_max_abs(const float *x, long long n, float *out, void *stream); /* :119 */
void launch_quant_f32_i8(const float *x, long long n, float scale, int8_t *q, void *stream); /* :120 */
void launch_relu_quant(const float *y, long long n, float scale, int8_t *q, void *stream); /* :121 */
void launch_dequant_i8_f32(const int8_t *q, long long n, float scale, float *x, void *stream); /* :122 */
void launch_add_scaled_i8(const int8_t *a, float sa, const int8_t *b, float sb, long long n,
                          float *out, void *stream);                         /* backend.rs:123 */
void launch_epilogue_f32(const int32_t *acc, int acc_ld, float scale, float *out, int c, int ho,
                         int wo, long long total, void *stream);             /* backend.rs:124 */
void launch_avgpool_hw(const float *x, int c, int hw, long long b, float *out, void *stream); /* :125 */
void launch_avgpool_hw_backward(const float *dy, int c, int hw, long long b, float *dx,
                                void *stream);                               /* backend.rs:126 */
void launch_mul_gate(const float *x, const float *gate, int c, int hw, long long n, float *out,
                     void *stream);                                          /* backend.rs:127 */
void launch_mask_relu_bwd(const float *y, const float *dy, long long n, float *dx, void *stream); /* :128 */
void launch_zero_f32(float *p, long long n, void *stream);                  /* backend.rs:129 */
void launch_transpose_i8(const int8_t *src, int rows, int cols, int8_t *dst, void *stream); /* :130 */
void launch_add_f32(const float *a, const float *b, long long n, float *o, void *stream); /* :131 */
void launch_mul_f32(const float *a, const float *b, long long n, float *o, void *stream); /* :132 */
void launch_meanpool_h(const float *x, int c, int h, int w, long long b, float *out,
                       void *stream);                                        /* backend.rs:133 */
void launch_meanpool_h_backward(const float *dy, int c, int h, int w, long long b, float *dx,
                                void *stream);                               /* backend.rs:134 */

/* ------------------------------------------------ workspace / device ---- */
void *trba_workspace_acquire(size_t bytes);                                  /* backend.rs:135 */
size_t trba_workspace_size(void);                                            /* backend.rs:136 */
void trba_workspace_release(void *ptr);                                      /* backend.rs:137 */
void trba_workspace_release_all(void);                                       /* backend.rs:138 */
const char *trba_backend_name(void);                                         /* backend.rs:139 */
const char *trba_device_name(void);                                          /* backend.rs:140 */
int trba_device_cc_major(void);                                              /* backend.rs:141 */
int trba_device_cc_minor(void);                                              /* backend.rs:142 */

/* ------------------------------------------------ static weight blobs --- */
void allocate_model_weights(size_t cnn_size, size_t bilstm_size, size_t attn_size,
                            size_t ctc_size);                                /* gpu_memory.rs:14 */
void upload_cnn_weights(const void *data, size_t size);                     /* gpu_memory.rs:15 */
void upload_bilstm_weights(const void *data, size_t size);                  /* gpu_memory.rs:16 */
void upload_attention_weights(const void *data, size_t size);               /* gpu_memory.rs:17 */
void upload_ctc_weights(const void *data, size_t size);                     /* gpu_memory.rs:18 */
void free_model_weights(void);                                               /* gpu_memory.rs:19 */
void *get_cnn_weights_ptr(void);
void *get_bilstm_weights_ptr(void);
void *get_attention_weights_ptr(void);
void *get_ctc_weights_ptr(void);

/* ------------------------------------- error reporting (new, no ref.) --- */
/* The reference aborts on every CUDA error (cuda/kernels.cu:37-50).  These
 * three let a caller keep the process alive and poll instead. */
void trba_set_abort_on_error(int on);
int trba_last_error(void);          /* 0 = no error since the last clear */
const char *trba_last_error_string(void);
void trba_clear_error(void);

#ifdef __cplusplus
}
#endif
#endif
