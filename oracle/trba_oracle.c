/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle of the TRBA INT8-QAT hot path.
 *
 * Restates, function by function, the reference's native backend ABI
 * (trba-rust src/backend.rs, later snapshot src/backend.rs:14-143) with the
 * arithmetic of its CPU mirror (cuda/cpu_backend.cpp of the later snapshot).
 * Each function cites the reference lines it follows.  "Device" pointers are
 * host pointers and the trailing stream argument is ignored.
 *
 * Summation order: where the reference accumulates in double per OpenMP
 * thread and then adds float partials, this restatement accumulates the whole
 * range in double and rounds once; results agree to float rounding, which is
 * the tolerance the parity tests state for those outputs.  Everything on the
 * integer / quantisation path (GEMM, im2col, epilogues, quantisers, pools)
 * is bit-exact with the reference.
 */
#include "trba_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef long long i64;

static inline int a16(int x) { return (x + 15) & ~15; }
static inline float fminf_(float a, float b) { return a < b ? a : b; }
static inline float fmaxf_(float a, float b) { return a > b ? a : b; }
static inline float clampf(float v, float lo, float hi) { return fminf_(fmaxf_(v, lo), hi); }

/* ---------------------------------------------------------------- det() -- */
/* src/tests.rs:39-43: x = (i*2654435761) ^ seed (wrapping, 64-bit);
 * x = x*6364136223846793005 + 1442695040888963407; ((x>>33) as f32)/2^31*2-1 */
float orc_det(unsigned long long i, unsigned long long seed) {
    unsigned long long x = (i * 2654435761ULL) ^ seed;
    x = x * 6364136223846793005ULL + 1442695040888963407ULL;
    float hi = (float)(x >> 33);
    return hi / 2147483648.0f * 2.0f - 1.0f;
}

void orc_det_fill(float *out, i64 n, unsigned long long seed, float mul) {
    for (i64 i = 0; i < n; ++i) out[i] = orc_det((unsigned long long)i, seed) * mul;
}

/* Rust `(det(i, seed) * mul) as i8`: truncation toward zero, saturating. */
void orc_det_fill_i8(int8_t *out, i64 n, unsigned long long seed, float mul) {
    for (i64 i = 0; i < n; ++i) {
        float v = orc_det((unsigned long long)i, seed) * mul;
        float t = truncf(v);
        if (t > 127.f) t = 127.f;
        if (t < -128.f) t = -128.f;
        out[i] = (int8_t)t;
    }
}

/* ================================================================ GEMMs == */
/* cpu_backend.cpp:93-112 — C[M,N] s32 = A[M,Kp] . B[N,Kp]^T over k < K. */
void launch_gemm_int8(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, void *s) {
    (void)s;
    if (M <= 0 || N <= 0 || K <= 0) return;
    const int Kp = a16(K);
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        const int8_t *a = A + (i64)m * Kp;
        for (int n = 0; n < N; ++n) {
            const int8_t *b = B + (i64)n * Kp;
            int32_t acc = 0;
            for (int k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
            C[(i64)m * N + n] = acc;
        }
    }
}

static float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u, e = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (e == 0) {
        if (man == 0) bits = sign << 31;
        else {
            e = 127 - 15 + 1;
            while ((man & 0x400u) == 0) { man <<= 1; --e; }
            man &= 0x3FFu;
            bits = (sign << 31) | (e << 23) | (man << 13);
        }
    } else if (e == 31) bits = (sign << 31) | 0x7F800000u | (man << 13);
    else bits = (sign << 31) | ((e + 127 - 15) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* cpu_backend.cpp:114-131 — f16 operands, same padding contract. */
void launch_gemm_fp16(const void *A, const void *B, float *C, int M, int N, int K, void *s) {
    (void)s;
    if (M <= 0 || N <= 0 || K <= 0) return;
    const int Kp = a16(K);
    const uint16_t *a = (const uint16_t *)A, *b = (const uint16_t *)B;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.f;
            for (int k = 0; k < K; ++k) acc += h2f(a[(i64)m * Kp + k]) * h2f(b[(i64)n * Kp + k]);
            C[(i64)m * N + n] = acc;
        }
}

/* cpu_backend.cpp:133-152 — C = A[M,K] . B[K,N], fp32. */
void launch_gemm_fp32(const float *A, const float *B, float *C, int M, int N, int K, void *s) {
    (void)s;
    if (M <= 0 || N <= 0 || K <= 0) return;
    for (int m = 0; m < M; ++m) {
        float *c = C + (i64)m * N;
        for (int n = 0; n < N; ++n) c[n] = 0.f;
        for (int k = 0; k < K; ++k) {
            const float av = A[(i64)m * K + k];
            if (av == 0.f) continue;
            for (int n = 0; n < N; ++n) c[n] += av * B[(i64)k * N + n];
        }
    }
}

/* ============================================================ epilogues == */
/* cpu_backend.cpp:157-181 — int8 = rint(clamp(max(acc/div + bias, 0) * mul)). */
void launch_conv_epilogue(const int32_t *acc, const float *bias, int8_t *out, int acc_ld,
                          float acc_div, float out_mul, int B, int C, int Ho, int Wo, void *s) {
    (void)s;
    const i64 hw = (i64)Ho * Wo, total = (i64)B * C * hw;
    for (i64 i = 0; i < total; ++i) {
        i64 b = i / ((i64)C * hw);
        int oc = (int)((i / hw) % C);
        i64 row = b * hw + (i % hw);
        float v = (float)acc[row * acc_ld + oc] / acc_div + bias[oc];
        v = fmaxf_(v, 0.0f) * out_mul;
        v = clampf(v, -127.0f, 127.0f);
        out[i] = (int8_t)lrintf(v);
    }
}

/* cpu_backend.cpp:858-868 — acc[row, oc] * scale -> NCHW fp32. */
void launch_epilogue_f32(const int32_t *acc, int acc_ld, float scale, float *out, int C, int Ho,
                         int Wo, i64 total, void *s) {
    (void)s;
    const i64 hw = (i64)Ho * Wo;
    for (i64 i = 0; i < total; ++i) {
        i64 b = i / ((i64)C * hw);
        int oc = (int)((i / hw) % C);
        i64 row = b * hw + (i % hw);
        out[i] = (float)acc[row * acc_ld + oc] * scale;
    }
}

/* =============================================================== im2col == */
/* cpu_backend.cpp:186-226 — rows (b,oh,ow), cols (c,kh,kw), ld col_ld, zero
 * tail columns and tail rows up to align16(rows). */
void launch_im2col_pad(const int8_t *input, int8_t *col, int batch, int C, int H, int W, int kH,
                       int kW, int sH, int sW, int pH, int pW, int Ho, int Wo, int col_ld, void *s) {
    (void)s;
    const int cols = C * kH * kW;
    const i64 rows = (i64)batch * Ho * Wo;
    if (col_ld < cols || (col_ld & 15) || rows <= 0) return;
    for (i64 row = 0; row < rows; ++row) {
        int b = (int)(row / ((i64)Ho * Wo));
        int rem = (int)(row - (i64)b * Ho * Wo);
        int oh = rem / Wo, ow = rem % Wo;
        int8_t *dst = col + row * col_ld;
        int p = 0;
        for (int ci = 0; ci < C; ++ci)
            for (int kh = 0; kh < kH; ++kh)
                for (int kw = 0; kw < kW; ++kw) {
                    int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
                    dst[p++] = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                                   ? input[((i64)(b * C + ci) * H + ih) * W + iw]
                                   : (int8_t)0;
                }
        for (; p < col_ld; ++p) dst[p] = 0;
    }
    const i64 rows_p = (rows + 15) / 16 * 16;
    if (rows_p > rows) memset(col + rows * col_ld, 0, (size_t)((rows_p - rows) * col_ld));
}

/* cpu_backend.cpp:228-256 — fp32 compact im2col. */
void launch_im2col_gpu(const int8_t *input, float *col, int batch, int C, int H, int W, int kH,
                       int kW, int sH, int sW, int pH, int pW, int Ho, int Wo, void *s) {
    (void)s;
    const int cols = C * kH * kW;
    const i64 rows = (i64)batch * Ho * Wo;
    for (i64 row = 0; row < rows; ++row) {
        int b = (int)(row / ((i64)Ho * Wo));
        int rem = (int)(row - (i64)b * Ho * Wo);
        int oh = rem / Wo, ow = rem % Wo, p = 0;
        for (int ci = 0; ci < C; ++ci)
            for (int kh = 0; kh < kH; ++kh)
                for (int kw = 0; kw < kW; ++kw) {
                    int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
                    col[row * cols + p++] = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                                                ? (float)input[((i64)(b * C + ci) * H + ih) * W + iw]
                                                : 0.0f;
                }
    }
}

/* ========================================================= conv backward == */
/* cpu_backend.cpp:261-293 — fp32 wgrad by direct sum (float accumulator). */
void launch_conv_backward_grad_weight(const int8_t *input, const float *go, float *gw, int B,
                                      int Cin, int H, int W, int Cout, int kH, int kW, int sH,
                                      int sW, int pH, int pW, int Ho, int Wo, void *s) {
    (void)s;
    if (B <= 0 || Cout <= 0 || Cin <= 0) return;
    const int cols = Cin * kH * kW, hwo = Ho * Wo;
    for (int oc = 0; oc < Cout; ++oc)
        for (int ci = 0; ci < cols; ++ci) {
            const int c = ci / (kH * kW), kk = ci % (kH * kW), kh = kk / kW, kw = kk % kW;
            float acc = 0.0f;
            for (int b = 0; b < B; ++b) {
                const int8_t *in_b = input + (i64)(b * Cin + c) * H * W;
                const float *go_b = go + (i64)(b * Cout + oc) * hwo;
                for (int p = 0; p < hwo; ++p) {
                    int oh = p / Wo, ow = p % Wo;
                    int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
                    if (ih >= 0 && ih < H && iw >= 0 && iw < W) acc += go_b[p] * (float)in_b[ih * W + iw];
                }
            }
            gw[(i64)oc * cols + ci] = acc;
        }
}

/* cpu_backend.cpp:295-313 */
void launch_conv_backward_grad_bias(const float *go, float *gb, int B, int Cout, int Ho, int Wo,
                                    void *s) {
    (void)s;
    if (B <= 0 || Cout <= 0) return;
    const i64 hw = (i64)Ho * Wo;
    for (int oc = 0; oc < Cout; ++oc) {
        float acc = 0.0f;
        for (int b = 0; b < B; ++b)
            for (i64 i = 0; i < hw; ++i) acc += go[((i64)b * Cout + oc) * hw + i];
        gb[oc] = acc;
    }
}

/* Shared dgrad gather of cpu_backend.cpp:315-397: for each input pixel, sum
 * over (kh, kw) taps that land on an output pixel, then over oc (in order). */
static void dgrad_gather(const float *go, const float *wf, const int8_t *wq, i64 w_ld, float w_scale,
                         float *gi, int B, int Cin, int H, int W, int Cout, int kH, int kW, int sH,
                         int sW, int pH, int pW, int Ho, int Wo) {
    const int hwo = Ho * Wo, hwi = H * W;
#pragma omp parallel for schedule(static)
    for (int b = 0; b < B; ++b) {
        const float *go_b = go + (i64)b * Cout * hwo;
        for (int ci = 0; ci < Cin; ++ci)
            for (int ih = 0; ih < H; ++ih)
                for (int iw = 0; iw < W; ++iw) {
                    float acc = 0.0f;
                    for (int kh = 0; kh < kH; ++kh) {
                        int nh = ih + pH - kh;
                        if (nh < 0 || nh % sH) continue;
                        int oh = nh / sH;
                        if (oh >= Ho) continue;
                        for (int kw = 0; kw < kW; ++kw) {
                            int nw = iw + pW - kw;
                            if (nw < 0 || nw % sW) continue;
                            int ow = nw / sW;
                            if (ow >= Wo) continue;
                            const i64 wc = (i64)(ci * kH + kh) * kW + kw;
                            const float *gp = go_b + oh * Wo + ow;
                            if (wq) {
                                for (int oc = 0; oc < Cout; ++oc)
                                    acc += gp[(i64)oc * hwo] * (float)wq[(i64)oc * w_ld + wc];
                            } else {
                                for (int oc = 0; oc < Cout; ++oc)
                                    acc += gp[(i64)oc * hwo] * wf[(i64)oc * w_ld + wc];
                            }
                        }
                    }
                    gi[((i64)(b * Cin + ci)) * hwi + ih * W + iw] = wq ? acc * w_scale : acc;
                }
    }
}

void launch_conv_backward_grad_input(const float *go, const float *Wt, float *gi, int B, int Cin,
                                     int H, int W, int Cout, int kH, int kW, int sH, int sW, int pH,
                                     int pW, int Ho, int Wo, void *s) {
    (void)s;
    if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0) return;
    dgrad_gather(go, Wt, NULL, (i64)Cin * kH * kW, 1.0f, gi, B, Cin, H, W, Cout, kH, kW, sH, sW, pH,
                 pW, Ho, Wo);
}

/* later snapshot cpu_backend.cpp:357-397 — int8 weights with ld w_ld, scale once. */
void launch_conv_backward_grad_input_i8(const float *go, const int8_t *Wq, int w_ld, float w_scale,
                                        float *gi, int B, int Cin, int H, int W, int Cout, int kH,
                                        int kW, int sH, int sW, int pH, int pW, int Ho, int Wo,
                                        void *s) {
    (void)s;
    if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0) return;
    dgrad_gather(go, NULL, Wq, w_ld, w_scale, gi, B, Cin, H, W, Cout, kH, kW, sH, sW, pH, pW, Ho, Wo);
}

/* ============================================================== maxpool == */
/* cpu_backend.cpp:399-415 */
void launch_maxpool2x2_backward(const float *go, const i64 *idx, float *gi, i64 out_n, i64 in_n,
                                void *s) {
    (void)s;
    memset(gi, 0, (size_t)in_n * sizeof(float));
    for (i64 i = 0; i < out_n; ++i) gi[idx[i]] += go[i];
}

void maxpool2x2_backward_host(const float *go, const unsigned long long *idx, float *gi,
                              unsigned long long out_n, unsigned long long in_n) {
    memset(gi, 0, (size_t)in_n * sizeof(float));
    for (unsigned long long i = 0; i < out_n; ++i) gi[idx[i]] += go[i];
}

/* later snapshot cpu_backend.cpp:498-522 — first strict maximum in
 * (0,0),(0,1),(1,0),(1,1) order. */
void launch_maxpool2x2_forward_i8(const int8_t *x, int8_t *y, int B, int C, int H, int W, void *s) {
    (void)s;
    if (B <= 0 || C <= 0 || H < 2 || W < 2 || (H & 1) || (W & 1)) {
        fprintf(stderr, "oracle maxpool2x2_forward_i8: bad shape\n");
        abort();
    }
    const int Ho = H / 2, Wo = W / 2;
    for (i64 bc = 0; bc < (i64)B * C; ++bc)
        for (int oh = 0; oh < Ho; ++oh)
            for (int ow = 0; ow < Wo; ++ow) {
                const int8_t *w = x + bc * H * W + (i64)(2 * oh) * W + 2 * ow;
                int8_t m = w[0];
                if (w[1] > m) m = w[1];
                if (w[W] > m) m = w[W];
                if (w[W + 1] > m) m = w[W + 1];
                y[bc * Ho * Wo + (i64)oh * Wo + ow] = m;
            }
}

/* later snapshot cpu_backend.cpp:524-554 — argmax recomputed from x. */
void launch_maxpool2x2_backward_i8(const int8_t *x, const float *dy, float *dx, int B, int C, int H,
                                   int W, void *s) {
    (void)s;
    if (B <= 0 || C <= 0 || H < 2 || W < 2 || (H & 1) || (W & 1)) {
        fprintf(stderr, "oracle maxpool2x2_backward_i8: bad shape\n");
        abort();
    }
    const int Ho = H / 2, Wo = W / 2;
    for (i64 bc = 0; bc < (i64)B * C; ++bc)
        for (int oh = 0; oh < Ho; ++oh)
            for (int ow = 0; ow < Wo; ++ow) {
                const i64 base = bc * H * W + (i64)(2 * oh) * W + 2 * ow;
                const int8_t *w = x + base;
                int win = 0;
                int8_t m = w[0];
                if (w[1] > m) { m = w[1]; win = 1; }
                if (w[W] > m) { m = w[W]; win = W; }
                if (w[W + 1] > m) { m = w[W + 1]; win = W + 1; }
                const float g = dy[bc * Ho * Wo + (i64)oh * Wo + ow];
                dx[base] = win == 0 ? g : 0.f;
                dx[base + 1] = win == 1 ? g : 0.f;
                dx[base + W] = win == W ? g : 0.f;
                dx[base + W + 1] = win == W + 1 ? g : 0.f;
            }
}

/* ================================================ device optimiser state == */
/* later snapshot cpu_backend.cpp:420-427 */
void launch_grad_accum_i32(const int32_t *acc, float *g, float scale, i64 n, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) g[i] += (float)acc[i] * scale;
}

/* later snapshot cpu_backend.cpp:429-438 */
void launch_sum_sq_add_f32(const float *x, double *out, i64 n, void *s) {
    (void)s;
    double acc = 0.0;
    for (i64 i = 0; i < n; ++i) acc += (double)x[i] * (double)x[i];
    *out += acc;
}

/* later snapshot cpu_backend.cpp:440-456 — Adam with f64 intermediates. */
void launch_adam_f32(float *p, const float *g, float *m, float *v, i64 n, double lr, double wd,
                     double clip, double b1, double b2, double eps, double bc1, double bc2, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) {
        const double gi = (double)(float)((double)g[i] * clip) + wd * (double)p[i];
        const float mf = (float)(b1 * (double)m[i] + (1.0 - b1) * gi);
        const float vf = (float)(b2 * (double)v[i] + (1.0 - b2) * gi * gi);
        m[i] = mf;
        v[i] = vf;
        const double mh = (double)mf / bc1, vh = (double)vf / bc2;
        p[i] -= (float)(lr * mh / (sqrt(vh) + eps));
    }
}

/* later snapshot cpu_backend.cpp:458-465 */
void launch_max_abs_f32(const float *x, float *out, i64 n, void *s) {
    (void)s;
    float mx = 0.0f;
    for (i64 i = 0; i < n; ++i) mx = fmaxf_(mx, fabsf(x[i]));
    *out = mx;
}

/* later snapshot cpu_backend.cpp:467-493 — s = max/127 in double (1 if 0),
 * q = round-half-away(clamp((float)(w/s as double))), zero-padded to
 * [align16(rows), kp]. */
void launch_quantize_pad_i8(const float *w, const float *max_abs, float *w_s_out, int8_t *wq,
                            i64 rows, i64 col, i64 kp, void *s) {
    (void)s;
    if (rows <= 0 || col <= 0) return;
    if (kp < col || (kp & 15) || !wq || !max_abs) {
        fprintf(stderr, "oracle quantize_pad_i8: bad args\n");
        abort();
    }
    const double mx = (double)*max_abs;
    const float sc = (float)(mx > 0.0 ? mx / 127.0 : 1.0);
    if (w_s_out) *w_s_out = sc;
    const i64 rp = (rows + 15) & ~15LL;
    for (i64 r = 0; r < rp; ++r)
        for (i64 c = 0; c < kp; ++c) {
            float v = 0.0f;
            if (r < rows && c < col) v = clampf((float)((double)w[r * col + c] / (double)sc), -127.f, 127.f);
            wq[r * kp + c] = (int8_t)roundf(v);
        }
}

/* later snapshot cpu_backend.cpp:1197-1213 — momentum-free Muon. */
void launch_muon_step_f32(float *w, const float *g, const double *gsq, i64 n, double lr, double wd,
                          double clip, double min_dim, double max_dim, double cap, i64 autoscale,
                          void *s) {
    (void)s;
    if (n <= 0 || !w || !g || !gsq) return;
    const double frob = sqrt(fmax(*gsq, 1e-30));
    const double scale = fmin(sqrt(min_dim) / fmax(frob, 1e-8), cap);
    const double lre = autoscale ? lr * sqrt(max_dim) : lr;
    const float step = (float)(clip * lre * scale);
    const float dec = (float)(1.0 - lr * wd);
    for (i64 i = 0; i < n; ++i) {
        const float u = w[i] * dec - step * g[i];
        w[i] = isfinite(u) ? u : 0.0f;
    }
}

/* ============================================================ utilities == */
void cuda_float_to_half(const float *src, void *dst, i64 n, void *s) {
    (void)s;
    uint16_t *d = (uint16_t *)dst;
    for (i64 i = 0; i < n; ++i) {
        uint32_t bits;
        memcpy(&bits, &src[i], 4);
        uint32_t sign = (bits >> 16) & 0x8000u;
        int32_t e = (int32_t)((bits >> 23) & 0xFFu) - 127 + 15;
        uint32_t man = bits & 0x7FFFFFu;
        if (e <= 0) d[i] = (uint16_t)sign;
        else if (e >= 31) d[i] = (uint16_t)(sign | 0x7C00u);
        else d[i] = (uint16_t)(sign | ((uint32_t)e << 10) | (man >> 13));
    }
}

void cuda_scale_vector(float *x, float scale, i64 n, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) x[i] *= scale;
}

void cuda_transpose_f32(const float *src, float *dst, int rows, int cols, void *s) {
    (void)s;
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < cols; ++j) dst[(i64)j * rows + i] = src[(i64)i * cols + j];
}

/* ======================================================= BN / quant ops == */
/* later snapshot cpu_backend.cpp:742-768 — per-channel sums, then
 * mean = s/count, var = max(sq/count - mean^2, 0) in float. */
void launch_bn_stats(const float *x, int B, int C, int HW, float *mean, float *var, void *s) {
    (void)s;
    const i64 n = (i64)B * C * HW, count = (i64)B * HW;
    if (n <= 0) return;
    for (int c = 0; c < C; ++c) {
        double sm = 0.0, sq = 0.0;
        for (int b = 0; b < B; ++b) {
            const float *p = x + ((i64)b * C + c) * HW;
            for (int j = 0; j < HW; ++j) {
                const double v = p[j];
                sm += v;
                sq += v * v;
            }
        }
        const float m = (float)sm / (float)count;
        const float v = (float)sq / (float)count - m * m;
        mean[c] = m;
        var[c] = v < 0.0f ? 0.0f : v;
    }
}

/* later snapshot cpu_backend.cpp:770-780 — ((x-mean)*r)*gamma + beta. */
void launch_bn_apply(const float *x, const float *mean, const float *var, const float *gamma,
                     const float *beta, float eps, float *y, int C, int HW, i64 n, void *s) {
    (void)s;
    float *r = (float *)malloc(sizeof(float) * (size_t)(C > 0 ? C : 1));
    for (int c = 0; c < C; ++c) r[c] = 1.0f / sqrtf(var[c] + eps);
    for (i64 i = 0; i < n; ++i) {
        const int c = (int)((i / HW) % C);
        y[i] = (x[i] - mean[c]) * r[c] * gamma[c] + beta[c];
    }
    free(r);
}

/* later snapshot cpu_backend.cpp:782-802 */
void launch_bn_bwd_sums(const float *dy, const float *x, const float *mean, const float *var,
                        float eps, int C, int HW, i64 n, float *sum_dy, float *sum_dy_xhat, void *s) {
    (void)s;
    double *sd = (double *)calloc((size_t)(C > 0 ? C : 1), sizeof(double));
    double *sx = (double *)calloc((size_t)(C > 0 ? C : 1), sizeof(double));
    float *r = (float *)malloc(sizeof(float) * (size_t)(C > 0 ? C : 1));
    for (int c = 0; c < C; ++c) r[c] = 1.0f / sqrtf(var[c] + eps);
    for (i64 i = 0; i < n; ++i) {
        const int c = (int)((i / HW) % C);
        const float xh = (x[i] - mean[c]) * r[c];
        sd[c] += dy[i];
        sx[c] += (double)(dy[i] * xh);
    }
    for (int c = 0; c < C; ++c) {
        sum_dy[c] = (float)sd[c];
        sum_dy_xhat[c] = (float)sx[c];
    }
    free(sd);
    free(sx);
    free(r);
}

/* later snapshot cpu_backend.cpp:804-817 */
void launch_bn_bwd_dx(const float *dy, const float *x, const float *mean, const float *var,
                      const float *gamma, const float *sum_dy, const float *sum_dy_xhat, float eps,
                      int C, int HW, i64 n, i64 count, float *dx, void *s) {
    (void)s;
    const float cnt = (float)count;
    for (i64 i = 0; i < n; ++i) {
        const int c = (int)((i / HW) % C);
        const float r = 1.0f / sqrtf(var[c] + eps);
        const float xh = (x[i] - mean[c]) * r;
        dx[i] = gamma[c] * r / cnt * (cnt * dy[i] - sum_dy[c] - xh * sum_dy_xhat[c]);
    }
}

/* later snapshot cpu_backend.cpp:819-827 */
void launch_reduce_max_abs(const float *x, i64 n, float *out, void *s) {
    (void)s;
    float m = 0.0f;
    for (i64 i = 0; i < n; ++i) {
        const float v = fabsf(x[i]);
        if (v > m) m = v;
    }
    *out = m;
}

/* later snapshot cpu_backend.cpp:829-836 — lrint (half to even) of clamp(x * (1/s)). */
void launch_quant_f32_i8(const float *x, i64 n, float scale, int8_t *q, void *s) {
    (void)s;
    const float inv = 1.0f / scale;
    for (i64 i = 0; i < n; ++i) q[i] = (int8_t)lrintf(clampf(x[i] * inv, -127.0f, 127.0f));
}

/* later snapshot cpu_backend.cpp:838-845 */
void launch_relu_quant(const float *y, i64 n, float scale, int8_t *q, void *s) {
    (void)s;
    const float inv = 1.0f / scale;
    for (i64 i = 0; i < n; ++i) q[i] = (int8_t)lrintf(fminf_(fmaxf_(y[i], 0.0f) * inv, 127.0f));
}

void launch_dequant_i8_f32(const int8_t *q, i64 n, float scale, float *x, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) x[i] = (float)q[i] * scale;
}

void launch_add_scaled_i8(const int8_t *a, float sa, const int8_t *b, float sb, i64 n, float *out,
                          void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) out[i] = (float)a[i] * sa + (float)b[i] * sb;
}

/* later snapshot cpu_backend.cpp:870-879 — mean over HW, double sum. */
void launch_avgpool_hw(const float *x, int C, int HW, i64 B, float *out, void *s) {
    (void)s;
    for (i64 i = 0; i < B * C; ++i) {
        double acc = 0.0;
        for (int j = 0; j < HW; ++j) acc += x[i * HW + j];
        out[i] = (float)(acc / HW);
    }
}

void launch_avgpool_hw_backward(const float *dy, int C, int HW, i64 B, float *dx, void *s) {
    (void)s;
    for (i64 i = 0; i < B * C; ++i) {
        const float v = dy[i] / (float)HW;
        for (int j = 0; j < HW; ++j) dx[i * HW + j] = v;
    }
}

void launch_mul_gate(const float *x, const float *gate, int C, int HW, i64 n, float *out, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) {
        const int c = (int)((i / HW) % C);
        const i64 b = i / ((i64)C * HW);
        out[i] = x[i] * gate[b * C + c];
    }
}

void launch_mask_relu_bwd(const float *y, const float *dy, i64 n, float *dx, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) dx[i] = y[i] > 0.0f ? dy[i] : 0.0f;
}

void launch_zero_f32(float *p, i64 n, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) p[i] = 0.0f;
}

void launch_transpose_i8(const int8_t *src, int rows, int cols, int8_t *dst, void *s) {
    (void)s;
    for (int c = 0; c < cols; ++c)
        for (int r = 0; r < rows; ++r) dst[(i64)c * rows + r] = src[(i64)r * cols + c];
}

void launch_add_f32(const float *a, const float *b, i64 n, float *o, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) o[i] = a[i] + b[i];
}

void launch_mul_f32(const float *a, const float *b, i64 n, float *o, void *s) {
    (void)s;
    for (i64 i = 0; i < n; ++i) o[i] = a[i] * b[i];
}

/* later snapshot cpu_backend.cpp:927-939 — [B,C,H,W] -> [B,W,C], float sum over h. */
void launch_meanpool_h(const float *x, int C, int H, int W, i64 B, float *out, void *s) {
    (void)s;
    for (i64 i = 0; i < B * W * C; ++i) {
        const int c = (int)(i % C), w = (int)((i / C) % W);
        const i64 b = i / ((i64)C * W);
        float acc = 0.0f;
        for (int h = 0; h < H; ++h) acc += x[((b * C + c) * H + h) * W + w];
        out[i] = acc / (float)H;
    }
}

void launch_meanpool_h_backward(const float *dy, int C, int H, int W, i64 B, float *dx, void *s) {
    (void)s;
    for (i64 i = 0; i < B * W * C; ++i) {
        const int c = (int)(i % C), w = (int)((i / C) % W);
        const i64 b = i / ((i64)C * W);
        const float v = dy[i] / (float)H;
        for (int h = 0; h < H; ++h) dx[((b * C + c) * H + h) * W + w] = v;
    }
}

/* ======================================================= BiLSTM (fp32) == */
/* later snapshot cpu_backend.cpp:983-1024 — one time slot of one direction;
 * x [B,T,D], gates [T,B,4H] post-activation, c/h [T,B,H] in slot order. */
static inline float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

void launch_lstm_fwd_step(const float *x, const float *w_ih, const float *b_ih, const float *w_hh,
                          const float *b_hh, float *gates, float *c_out, float *h_out, i64 B, i64 T,
                          i64 D, i64 H, i64 slot, i64 rev, void *s) {
    (void)s;
    if (B <= 0 || T <= 0 || D <= 0 || H <= 0 || slot < 0 || slot >= T) return;
    const i64 tt = rev ? T - 1 - slot : slot;
    for (i64 w = 0; w < B * H; ++w) {
        const i64 bi = w / H, i = w % H;
        const float *xr = x + (bi * T + tt) * D;
        float g[4];
        for (int q = 0; q < 4; ++q) {
            const i64 o = q * H + i;
            float acc = b_ih[o] + b_hh[o];
            for (i64 k = 0; k < D; ++k) acc += xr[k] * w_ih[o * D + k];
            if (slot) {
                const float *hp = h_out + ((slot - 1) * B + bi) * H;
                for (i64 k = 0; k < H; ++k) acc += hp[k] * w_hh[o * H + k];
            }
            g[q] = acc;
        }
        const float ig = sigm(g[0]), fg = sigm(g[1]), cg = tanhf(g[2]), og = sigm(g[3]);
        const float cp = slot ? c_out[((slot - 1) * B + bi) * H + i] : 0.0f;
        const float cn = fg * cp + ig * cg;
        const i64 gs = (slot * B + bi) * 4 * H, cs = (slot * B + bi) * H;
        gates[gs + i] = ig;
        gates[gs + H + i] = fg;
        gates[gs + 2 * H + i] = cg;
        gates[gs + 3 * H + i] = og;
        c_out[cs + i] = cn;
        h_out[cs + i] = og * tanhf(cn);
    }
}

/* later snapshot cpu_backend.cpp:1026-1051 */
void launch_lstm_bwd_cell(const float *dh_out, const float *gates, const float *ctrace,
                          const float *dh_next, const float *dc_next, float *dgates,
                          float *dc_next_out, i64 B, i64 H, i64 slot, void *s) {
    (void)s;
    if (B <= 0 || H <= 0) return;
    for (i64 idx = 0; idx < B * H; ++idx) {
        const i64 bi = idx / H, i = idx % H;
        const i64 cs = (slot * B + bi) * H, gs = (slot * B + bi) * 4 * H;
        const float cp = slot ? ctrace[((slot - 1) * B + bi) * H + i] : 0.0f;
        const float ig = gates[gs + i], fg = gates[gs + H + i], cg = gates[gs + 2 * H + i],
                    og = gates[gs + 3 * H + i];
        const float tc = tanhf(ctrace[cs + i]);
        const float dh = dh_out[cs + i] + dh_next[bi * H + i];
        const float dc = dh * og * (1.0f - tc * tc) + dc_next[bi * H + i] * fg;
        dgates[gs + i] = dc * cg * ig * (1.0f - ig);
        dgates[gs + H + i] = dc * cp * fg * (1.0f - fg);
        dgates[gs + 2 * H + i] = dc * ig * (1.0f - cg * cg);
        dgates[gs + 3 * H + i] = dh * tc * og * (1.0f - og);
        dc_next_out[bi * H + i] = dc;
    }
}

/* later snapshot cpu_backend.cpp:1053-1090 — dx[:,tt,:] = dgates W_ih, dh = dgates W_hh. */
void launch_lstm_bwd_rec(const float *dgates, const float *w_ih, const float *w_hh, float *dx,
                         float *dh_next, i64 B, i64 T, i64 D, i64 H, i64 slot, i64 rev, void *s) {
    (void)s;
    if (B <= 0 || T <= 0 || D <= 0 || H <= 0) return;
    const i64 tt = rev ? T - 1 - slot : slot;
    for (i64 bi = 0; bi < B; ++bi) {
        const float *dg = dgates + (slot * B + bi) * 4 * H;
        for (i64 k = 0; k < D; ++k) {
            float acc = 0.0f;
            for (i64 o = 0; o < 4 * H; ++o) acc += dg[o] * w_ih[o * D + k];
            dx[(bi * T + tt) * D + k] = acc;
        }
        for (i64 k = 0; k < H; ++k) {
            float acc = 0.0f;
            for (i64 o = 0; o < 4 * H; ++o) acc += dg[o] * w_hh[o * H + k];
            dh_next[bi * H + k] = acc;
        }
    }
}

/* later snapshot cpu_backend.cpp:1112-1139 — sum over (slot, b) of dgates x. */
void launch_lstm_wgrad_ih(const float *dgates, const float *x, float *g_w, i64 B, i64 T, i64 D, i64 H,
                          i64 rev, i64 accumulate, void *s) {
    (void)s;
    if (B <= 0 || T <= 0 || D <= 0 || H <= 0) return;
    for (i64 o = 0; o < 4 * H; ++o)
        for (i64 k = 0; k < D; ++k) {
            float acc = 0.0f;
            for (i64 j = 0; j < T * B; ++j) {
                const i64 slot = j / B, bi = j % B, tt = rev ? T - 1 - slot : slot;
                acc += dgates[j * 4 * H + o] * x[(bi * T + tt) * D + k];
            }
            if (accumulate) g_w[o * D + k] += acc;
            else g_w[o * D + k] = acc;
        }
}

/* later snapshot cpu_backend.cpp:1141-1169 — slot 0 has no previous h. */
void launch_lstm_wgrad_hh(const float *dgates, const float *htrace, float *g_w, i64 B, i64 T, i64 H,
                          i64 accumulate, void *s) {
    (void)s;
    if (B <= 0 || T <= 0 || H <= 0) return;
    for (i64 o = 0; o < 4 * H; ++o)
        for (i64 k = 0; k < H; ++k) {
            float acc = 0.0f;
            for (i64 j = B; j < T * B; ++j) {
                const i64 slot = j / B, bi = j % B;
                acc += dgates[j * 4 * H + o] * htrace[((slot - 1) * B + bi) * H + k];
            }
            if (accumulate) g_w[o * H + k] += acc;
            else g_w[o * H + k] = acc;
        }
}

/* later snapshot cpu_backend.cpp:1171-1194 */
void launch_lstm_bgrad(const float *dgates, float *g_b_ih, float *g_b_hh, i64 B, i64 T, i64 H,
                       i64 accumulate, void *s) {
    (void)s;
    if (B <= 0 || T <= 0 || H <= 0) return;
    for (i64 o = 0; o < 4 * H; ++o) {
        float acc = 0.0f;
        for (i64 j = 0; j < T * B; ++j) acc += dgates[j * 4 * H + o];
        if (accumulate) { g_b_ih[o] += acc; g_b_hh[o] += acc; }
        else { g_b_ih[o] = acc; g_b_hh[o] = acc; }
    }
}

/* ============================================================ plumbing == */
/* later snapshot cpu_backend.cpp:588-728: host memory stands in for device
 * memory; streams are no-ops. */
void cuda_malloc(void **p, size_t n) {
    *p = n ? calloc(1, n) : NULL;
}
void cuda_free(void *p) { free(p); }
void cuda_memcpy_h2d(void *d, const void *s, size_t n, void *st) { (void)st; if (n) memcpy(d, s, n); }
void cuda_memcpy_d2h(void *d, const void *s, size_t n, void *st) { (void)st; if (n) memcpy(d, s, n); }
void cuda_memcpy_dtod(void *d, const void *s, size_t n, void *st) { (void)st; if (n) memcpy(d, s, n); }
void cuda_sync(void *st) { (void)st; }
void cuda_stream_create(void **st) { *st = NULL; }
void cuda_stream_destroy(void *st) { (void)st; }
void cuda_get_memory_info(size_t *f, size_t *t) { if (f) *f = 0; if (t) *t = 0; }
const char *trba_backend_name(void) { return "oracle-cpu"; }
const char *trba_device_name(void) { return "CPU oracle"; }
int trba_device_cc_major(void) { return 0; }
int trba_device_cc_minor(void) { return 0; }
