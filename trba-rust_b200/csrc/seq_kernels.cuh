// Kernels of the sequence head of the device-resident QAT step: fp32 GEMM,
// BiLSTM recurrences, the attention decoder, CE and CTC losses.  All traces
// of the recurrences are kept per sample in time-position order [B, T, .].
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace trba {
namespace seq {

// C[m, n] = (float)(sum_k A(m, k) B(k, n)) [+ C[m, n] if accumulate] [+ bias[n]],
// A(m, k) = A[m*sam + k*sak], B(k, n) = B[k*sbk + n*sbn], C[m*ldc + n].
// The sum is accumulated in f64 and rounded once (the correctly rounded dot
// product in practice), so the result does not depend on the summation
// order; long K is split over CTAs through the f64 workspace `ws` and the
// partial sums are combined in a fixed order (deterministic).
struct Gemm {
    int M, N, K;
    const float *A;
    i64 sam, sak;
    const float *B;
    i64 sbk, sbn;
    float *C;
    i64 ldc;
    bool accumulate = false;
    const float *bias = nullptr;
    double *ws = nullptr;   // split-K workspace (may be null: no split)
    i64 ws_elems = 0;
};
void sgemm(const Gemm &g, cudaStream_t st);

// LSTM recurrences over all T slots (src/rnn.rs:107-166), the directions of
// a layer in one launch (grid y = entry of `dirs`).  Per direction: xg =
// x W_ih^T [B, T, 4H]; writes gates (post-activation) and c [B, T, .], h
// into cat[b, tt, dir*H + i] (row stride 2H) and h_prev [B, T, H].
struct LstmFwdDir {
    const float *xg, *b_ih, *b_hh, *w_hh;
    float *gates, *c, *h_prev;
    int rev, dir;
};
void lstm_fwd(const LstmFwdDir *dirs, int ndir, int B, int T, int H, float *cat, cudaStream_t st);
// Backward through time (src/rnn.rs:200-288), the directions in one launch:
// dh_out from dcat[b, tt, dir*H + i]; writes dgates [B, T, 4H].
struct LstmBwdDir {
    const float *gates, *c, *w_hh;
    float *dgates;
    int rev, dir;
};
void lstm_bwd(const LstmBwdDir *dirs, int ndir, const float *dcat, int B, int T, int H, cudaStream_t st);

// Attention decoder, teacher forced (src/attn.rs:119-261).  bh/proj_h [B,T,H];
// text_in [B, steps]; traces laid out [steps, B, .].
struct AttnFwd {
    const float *bh, *proj_h;
    const int32_t *text_in;
    const float *h2h_w, *h2h_b, *score_w, *w_ih, *b_ih, *w_hh, *b_hh;
    int B, T, H, V, steps;
    float *tanh_tr;  // [steps, B, T, H]
    float *alpha;    // [steps, B, T]
    float *cell_in;  // [steps, B, H+V]  (context, then the one-hot token)
    float *gates;    // [steps, B, 4H]
    float *hs, *cs;  // [steps, B, H]
    // greedy decoding only (attn_decode): generator, start token, output
    const float *gen_w = nullptr, *gen_b = nullptr;  // [V, H], [V]
    int sos = 1;
    int32_t *step_tokens = nullptr;  // [steps, B]: argmax token of every step
};
void attn_fwd(const AttnFwd &a, cudaStream_t st);
// Greedy decoding (src/attn.rs:368-447) over every step; the caller applies
// the reference's stop rule (all samples at eos) to step_tokens.
void attn_decode(const AttnFwd &a, cudaStream_t st);

// Backward (src/attn.rs:263-500): d_out_hid [steps, B, H]; writes dgates
// [steps, B, 4H], de [steps, B, T], dprojhh [steps, B, H], d_proj_h [B, T, H]
// and d_bh [B, T, H] (the context part only; the i2h path is added later).
struct AttnBwd {
    const float *d_out_hid, *bh, *tanh_tr, *alpha, *gates, *cs, *score_w, *w_ih, *w_hh, *h2h_w;
    int B, T, H, V, steps;
    float *dgates, *de, *dprojhh, *d_proj_h, *d_bh;
};
void attn_bwd(const AttnBwd &a, cudaStream_t st);

// CE with ignore-pad over logits [steps, B, V] (src/main.rs:2300-2328):
// d_logits = (p - onehot), row loss -ln p_tgt; rows whose target is pad get 0.
void ce_rows(const float *logits, const int32_t *target, int B, int steps, int V, int pad, float *d_logits,
             float *row_loss, cudaStream_t st);
// CTC (src/ctc.rs:103-193) over logits [B*T, V]; ctc_tgt [B, Lmax] with
// lengths ctc_len [B]; grad already multiplied by cw.
void ctc(const float *logits, const int32_t *ctc_tgt, const int32_t *ctc_len, int Lmax, int B, int T, int V,
         float cw, float *grad, double *sample_loss, cudaStream_t st);
// Column sums of X [rows, cols] (row stride ld) through sgemm with a ones
// vector `ones` (length >= rows): out[n] (+)= sum_r X[r*ld + n].
void col_sums(const float *X, int rows, int cols, i64 ld, const float *ones, float *out, bool accumulate,
              double *ws, i64 ws_elems, cudaStream_t st);
// Totals: attn = sum(row_loss)/count, ctc = sum(sample_loss)/n, loss =
// (1-cw) attn + cw ctc into out[0..2]; scales d_logits by (1-cw)/count.
void loss_finalize(const float *row_loss, const int32_t *target, int B, int steps, int pad, const double *sample_loss,
                   const int32_t *ctc_len, int T, float cw, float *d_logits, int V, float *out, cudaStream_t st);

}  // namespace seq
}  // namespace trba
