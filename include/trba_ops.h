/* INT8 operator API of libtrba_b200: device-resident counterparts of the
 * reference's LinearInt8 (src/linear.rs) and LSTMInt8 / BiLSTMInt8
 * (src/bilstm.rs).
 *
 * The reference keeps the f32 master weights and their int8 copies in host
 * vectors and moves every operand through a fresh device workspace per call.
 * Here each operator owns its master weights, int8 copies (already padded to
 * the tensor-core GEMM's [align16 rows, align16 k] layout) and scratch in
 * device memory; the *_host variants take host buffers like the Rust
 * methods, the others take device pointers and a stream.
 *
 * Errors follow the library policy (trba_last_error / abort on error);
 * functions returning int give 0 on success, -1 on a bad argument. */
#ifndef TRBA_OPS_H
#define TRBA_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* LSTMInt8::gemm_int8 (src/bilstm.rs:132-173): C s32 [m, n] = A [m, k] .
 * B [n, k]^T on compact (unpadded) device operands; pads internally. */
int trba_gemm_int8_compact(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k, void *stream);

/* ---- LinearInt8 (src/linear.rs:12-180) ---- */
typedef struct trba_linear_int8 trba_linear_int8;
/* LinearInt8::new with injected weights: weight_f32 [out, in] row-major
 * (host), bias [out] (host, NULL = zeros).  Quantises like
 * LinearInt8::quantize (src/linear.rs:53-59). */
trba_linear_int8 *trba_linear_int8_create(int in_features, int out_features, const float *weight_f32,
                                          const float *bias);
void trba_linear_int8_destroy(trba_linear_int8 *l);
/* LinearInt8::requantize (src/linear.rs:61-63). */
int trba_linear_int8_requantize(trba_linear_int8 *l, void *stream);
/* LinearInt8::forward (src/linear.rs:66-115): inp [rows, in] int8 ->
 * out [rows, out] int32; device pointers.  rows <= 0 is the reference's
 * assertion failure. */
int trba_linear_int8_forward(trba_linear_int8 *l, const int8_t *inp, int rows, int32_t *out, void *stream);
/* Same with host buffers; inp_len must be a positive multiple of in. */
int trba_linear_int8_forward_host(trba_linear_int8 *l, const int8_t *inp, long long inp_len, int32_t *out);
/* LinearInt8::backward (src/linear.rs:121-175): batch-averaged f32 outer
 * product, global-norm clip at 10, SGD step lr*clip, non-finite -> 0,
 * re-quantise.  inp [rows, in] and grad_out [rows, out] f32 on the device.
 * Returns the clip factor (0 when rows == 0); synchronises the stream. */
float trba_linear_int8_backward(trba_linear_int8 *l, const float *inp, const float *grad_out, int rows, float lr,
                                float mom, void *stream);
/* Same with host buffers and the reference's length rules (rows =
 * inp_len / in; 0 returned when rows == 0 or grad_len < rows * out). */
float trba_linear_int8_backward_host(trba_linear_int8 *l, const float *inp, long long inp_len,
                                     const float *grad_out, long long grad_len, float lr, float mom);
/* Host copies of the state (any pointer may be NULL): weight_f32 [out*in],
 * weight_int8 [out*in] (compact), bias [out], grad_f32 [out*in]. */
int trba_linear_int8_get(trba_linear_int8 *l, float *weight_f32, int8_t *weight_int8, float *bias,
                         float *grad_f32);
/* Replace the f32 weights / bias from the host (NULL = keep) and re-quantise. */
int trba_linear_int8_set(trba_linear_int8 *l, const float *weight_f32, const float *bias);
long long trba_linear_int8_param_count(const trba_linear_int8 *l);

/* ---- LSTMInt8 (src/bilstm.rs:13-178) ---- */
typedef struct trba_lstm_int8 trba_lstm_int8;
/* LSTMInt8::new with injected weights (host): w_ih [4H, input], w_hh
 * [4H, H], bias [4H] (NULL = zeros); gate order i, f, g, o. */
trba_lstm_int8 *trba_lstm_int8_create(int input_size, int hidden_size, const float *w_ih, const float *w_hh,
                                      const float *bias);
void trba_lstm_int8_destroy(trba_lstm_int8 *l);
int trba_lstm_int8_requantize(trba_lstm_int8 *l, void *stream);
/* LSTMInt8::forward_step (src/bilstm.rs:72-117): x [batch, input] int8,
 * h_prev / c_prev [batch, H] f32 -> h_new / c_new; device pointers.  h is
 * quantised with the fixed activation scale 10 before the h GEMM. */
int trba_lstm_int8_forward_step(trba_lstm_int8 *l, const int8_t *x, const float *h_prev, const float *c_prev,
                                int batch, float *h_new, float *c_new, void *stream);
/* LSTMInt8::i2h_forward / h2h_forward (src/bilstm.rs:119-127): s32 gate
 * projections [batch, 4H]. */
int trba_lstm_int8_i2h_forward(trba_lstm_int8 *l, const int8_t *x, int batch, int32_t *out, void *stream);
int trba_lstm_int8_h2h_forward(trba_lstm_int8 *l, const int8_t *h, int batch, int32_t *out, void *stream);
/* Host copies of the state (any pointer may be NULL). */
int trba_lstm_int8_get(trba_lstm_int8 *l, float *w_ih, int8_t *w_ih_int8, float *w_hh, int8_t *w_hh_int8,
                       float *bias);
long long trba_lstm_int8_param_count(const trba_lstm_int8 *l);

/* BiLSTMInt8::forward (src/bilstm.rs:195-251): x_seq [seq_len, batch,
 * input] int8 -> out [batch, 2H], each direction's hidden state averaged
 * over time.  Both directions step through time in forward order, as the
 * reference does.  Device pointers. */
int trba_bilstm_int8_forward(trba_lstm_int8 *fwd, trba_lstm_int8 *bwd, const int8_t *x_seq, int batch,
                             int seq_len, float *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif
