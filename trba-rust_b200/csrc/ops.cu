// INT8 operator API (include/trba_ops.h): LinearInt8 (src/linear.rs) and
// LSTMInt8 / BiLSTMInt8 (src/bilstm.rs) with device-resident state.
//
// Forward GEMMs run on the tcgen05 int8 GEMM behind launch_gemm_int8; the
// operands are kept (weights) or staged (activations) in its padded
// [align16 rows, align16 k] layout.  Float arithmetic follows the Rust code
// operation by operation (f32, no contraction): quantisation
// round(clamp(w / s, +-127)) with half-away rounding; the LSTM cell
// pre = (gi + gh) * (1/1270) + b, sigmoid = 1 / (1 + exp(-x)); the linear
// backward's batch sums run over rows in order.  exp and tanh are evaluated
// in f64 and rounded once.
#include <cuda_runtime.h>
#include <math.h>

#include <vector>

#include "common.cuh"
#include "trba_backend.h"
#include "trba_ops.h"

namespace trba {
namespace {

inline int a16(int x) { return (x + 15) & ~15; }

constexpr float kAccDivisor = 127.0f;       // src/conv2d.rs:24
constexpr float kActivationScale = 10.0f;   // src/bilstm.rs:29
constexpr float kLinearMaxGrad = 10.0f;     // src/linear.rs:152

// Device buffer that only grows.
template <class T>
struct DBuf {
    T *p = nullptr;
    size_t n = 0;
    bool ensure(size_t want) {
        if (want <= n) return true;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        if (cudaMalloc(&p, want * sizeof(T)) != cudaSuccess) {
            report_error(__FILE__, __LINE__, "operator scratch: cudaMalloc failed", -1);
            return false;
        }
        n = want;
        return true;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

// ---------------------------------------------------------------- kernels --

// dst [a16(m), a16(k)] = src [m, k] zero-padded.
__global__ void pad_i8_kernel(const int8_t *__restrict__ src, int8_t *__restrict__ dst, int m, int k, int ldd,
                              i64 total) {
    GRID_LOOP(i, total) {
        const i64 r = i / ldd;
        const int c = (int)(i - r * ldd);
        dst[i] = (r < m && c < k) ? src[r * k + c] : (int8_t)0;
    }
}

// max |w| over finite-or-not values, NaN ignored (Rust f32::max).
__global__ void absmax_kernel(const float *__restrict__ w, i64 n, unsigned *__restrict__ out) {
    float m = 0.0f;
    GRID_LOOP(i, n) {
        const float a = fabsf(w[i]);
        if (a > m) m = a;  // false for NaN
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

__device__ __forceinline__ int8_t round_clamp_i8(float v) {
    // Rust `v.clamp(-127, 127).round() as i8`: NaN -> 0
    if (v != v) return 0;
    v = fminf(fmaxf(v, -127.0f), 127.0f);
    return (int8_t)(int)roundf(v);
}

// LinearInt8::quantize (src/linear.rs:53-59) into the padded [a16 rows,
// a16 cols] operand.
__global__ void quantize_pad_kernel(const float *__restrict__ w, const unsigned *__restrict__ amax, int rows,
                                    int cols, int ld, i64 total, int8_t *__restrict__ q) {
    const float mx = __uint_as_float(*amax);
    const float s = mx > 0.0f ? fdiv(mx, 127.0f) : 1.0f;
    GRID_LOOP(i, total) {
        const i64 r = i / ld;
        const int c = (int)(i - r * ld);
        q[i] = (r < rows && c < cols) ? round_clamp_i8(fdiv(w[r * cols + c], s)) : (int8_t)0;
    }
}

// grad[o, i] = (sum_r go[r, o] * inp[r, i]) * inv_rows, f32, r in order
// (src/linear.rs:133-144).
__global__ void linear_wgrad_kernel(const float *__restrict__ inp, const float *__restrict__ go, int rows, int fi,
                                    int fo, float inv_rows, float *__restrict__ grad, double *__restrict__ sumsq) {
    double local = 0.0;
    GRID_LOOP(e, (i64)fo * fi) {
        const int o = (int)(e / fi), i = (int)(e - (i64)o * fi);
        float acc = 0.0f;
        for (int r = 0; r < rows; ++r) acc = fadd(acc, fmul(go[(i64)r * fo + o], inp[(i64)r * fi + i]));
        const float g = fmul(acc, inv_rows);
        grad[e] = g;
        const float g2 = fmul(g, g);
        local += (double)g2;
    }
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(sumsq, local);
}

// clip = norm > 10 ? 10 / norm : 1; step = lr * clip (src/linear.rs:146-154).
__global__ void linear_clip_kernel(const double *__restrict__ sumsq, float lr, float *__restrict__ out) {
    const float norm = sqrtf((float)*sumsq);
    const float clip = norm > kLinearMaxGrad ? fdiv(kLinearMaxGrad, norm) : 1.0f;
    out[0] = clip;
    out[1] = fmul(lr, clip);
}

// w = w - step * g, non-finite -> 0 (src/linear.rs:156-162).
__global__ void linear_update_kernel(float *__restrict__ w, const float *__restrict__ g, i64 n,
                                     const float *__restrict__ clip_step) {
    const float step = clip_step[1];
    GRID_LOOP(i, n) {
        const float u = fsub(w[i], fmul(step, g[i]));
        w[i] = isfinite(u) ? u : 0.0f;
    }
}

// bias[o] -= step * (sum_r go[r, o]) * inv_rows (src/linear.rs:164-171).
__global__ void linear_bias_kernel(float *__restrict__ bias, const float *__restrict__ go, int rows, int fo,
                                   float inv_rows, const float *__restrict__ clip_step) {
    const float step = clip_step[1];
    GRID_LOOP(o, fo) {
        float gb = 0.0f;
        for (int r = 0; r < rows; ++r) gb = fadd(gb, go[(i64)r * fo + o]);
        const float u = fsub(bias[o], fmul(fmul(step, gb), inv_rows));
        bias[o] = isfinite(u) ? u : 0.0f;
    }
}

// h_q [a16(batch), a16(H)] = round(clamp(h * 10, +-127)) (src/bilstm.rs:84-87).
__global__ void quantize_h_kernel(const float *__restrict__ h, int batch, int H, int ld, i64 total,
                                  int8_t *__restrict__ q) {
    GRID_LOOP(i, total) {
        const i64 r = i / ld;
        const int c = (int)(i - r * ld);
        q[i] = (r < batch && c < H) ? round_clamp_i8(fmul(h[r * H + c], kActivationScale)) : (int8_t)0;
    }
}

__device__ __forceinline__ float sigmoid_rs(float x) {
    return fdiv(1.0f, fadd(1.0f, (float)exp(-(double)x)));
}

// The LSTM cell of forward_step (src/bilstm.rs:99-115); gi / gh s32 [batch, 4H].
// With hsum != null, hsum += h_new (the time average of BiLSTMInt8::forward).
__global__ void lstm_cell_kernel(const int32_t *__restrict__ gi, const int32_t *__restrict__ gh,
                                 const float *__restrict__ bias, const float *__restrict__ c_prev, int batch, int H,
                                 float *__restrict__ h_new, float *__restrict__ c_new, float *__restrict__ hsum) {
    const float inv = fdiv(1.0f, kAccDivisor * kActivationScale);
    GRID_LOOP(e, (i64)batch * H) {
        const int b = (int)(e / H), i = (int)(e - (i64)b * H);
        const i64 row = (i64)b * 4 * H;
        float pre[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const i64 k = row + (i64)g * H + i;
            pre[g] = fadd(fmul(fadd((float)gi[k], (float)gh[k]), inv), bias[g * H + i]);
        }
        const float ig = sigmoid_rs(pre[0]), fg = sigmoid_rs(pre[1]), og = sigmoid_rs(pre[3]);
        const float cg = (float)tanh((double)pre[2]);
        const float c = fadd(fmul(fg, c_prev[e]), fmul(ig, cg));
        const float h = fmul(og, (float)tanh((double)c));
        c_new[e] = c;
        h_new[e] = h;
        if (hsum) hsum[e] = fadd(hsum[e], h);
    }
}

// out[b, d*H + i] = hsum_d[b, i] * inv_t (src/bilstm.rs:233-249).
__global__ void bilstm_out_kernel(const float *__restrict__ sf, const float *__restrict__ sb, int batch, int H,
                                  float inv_t, float *__restrict__ out) {
    GRID_LOOP(e, (i64)batch * H) {
        const int b = (int)(e / H), i = (int)(e - (i64)b * H);
        out[(i64)b * 2 * H + i] = fmul(sf[e], inv_t);
        out[(i64)b * 2 * H + H + i] = fmul(sb[e], inv_t);
    }
}

// ----------------------------------------------------------------- helpers --

void pad_i8(const int8_t *src, int8_t *dst, int m, int k, cudaStream_t st) {
    const int ld = a16(k);
    const i64 total = (i64)a16(m) * ld;
    pad_i8_kernel<<<grid_for(total), 256, 0, st>>>(src, dst, m, k, ld, total);
    TRBA_LAUNCH_CHECK();
}

void quantize_into(const float *w, int rows, int cols, unsigned *amax, int8_t *q, cudaStream_t st) {
    const i64 n = (i64)rows * cols;
    TRBA_CHECK(cudaMemsetAsync(amax, 0, sizeof(unsigned), st));
    absmax_kernel<<<grid_for(n), 256, 0, st>>>(w, n, amax);
    TRBA_LAUNCH_CHECK();
    const int ld = a16(cols);
    const i64 total = (i64)a16(rows) * ld;
    quantize_pad_kernel<<<grid_for(total), 256, 0, st>>>(w, amax, rows, cols, ld, total, q);
    TRBA_LAUNCH_CHECK();
}

// Compact [rows, cols] int8 out of the padded operand (host copy).
bool unpad_to_host(const int8_t *dpad, int rows, int cols, int8_t *host) {
    std::vector<int8_t> tmp((size_t)a16(rows) * a16(cols));
    if (cudaMemcpy(tmp.data(), dpad, tmp.size(), cudaMemcpyDeviceToHost) != cudaSuccess) return false;
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) host[(size_t)r * cols + c] = tmp[(size_t)r * a16(cols) + c];
    return true;
}

template <class T>
bool upload(T *dst, const T *host, size_t n) {
    return cudaMemcpy(dst, host, n * sizeof(T), cudaMemcpyHostToDevice) == cudaSuccess;
}

}  // namespace
}  // namespace trba

using namespace trba;

struct trba_linear_int8 {
    int in = 0, out = 0;
    float *w = nullptr, *bias = nullptr, *grad = nullptr;
    int8_t *wq = nullptr;  // [a16(out), a16(in)]
    unsigned *amax = nullptr;
    double *sumsq = nullptr;
    float *clip = nullptr;  // clip, step
    DBuf<int8_t> a_pad;
    DBuf<int8_t> in_stage;
    DBuf<int32_t> out_stage;
    DBuf<float> f_stage;
};

struct trba_lstm_int8 {
    int in = 0, H = 0;
    float *w_ih = nullptr, *w_hh = nullptr, *bias = nullptr;
    int8_t *q_ih = nullptr, *q_hh = nullptr;  // padded
    unsigned *amax = nullptr;
    DBuf<int8_t> x_pad, h_pad;
    DBuf<int32_t> gi, gh;
    DBuf<float> state;  // h, c ping-pong + sums
};

extern "C" {

int trba_gemm_int8_compact(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0 || !a || !b || !c) return -1;
    cudaStream_t st = as_stream(stream);
    const size_t na = (size_t)a16(m) * a16(k), nb = (size_t)a16(n) * a16(k);
    int8_t *buf = nullptr;
    TRBA_CHECK(cudaMallocAsync((void **)&buf, na + nb, st));
    if (!buf) return -1;
    pad_i8(a, buf, m, k, st);
    pad_i8(b, buf + na, n, k, st);
    launch_gemm_int8(buf, buf + na, c, m, n, k, stream);
    TRBA_CHECK(cudaFreeAsync(buf, st));
    return 0;
}

// ------------------------------------------------------------ LinearInt8 --
trba_linear_int8 *trba_linear_int8_create(int in_features, int out_features, const float *weight_f32,
                                          const float *bias) {
    TRBA_REQUIRE_RET(in_features > 0 && out_features > 0 && weight_f32, "trba_linear_int8_create: bad arguments",
                     nullptr);
    auto *l = new trba_linear_int8;
    l->in = in_features;
    l->out = out_features;
    const size_t nw = (size_t)in_features * out_features;
    bool ok = cudaMalloc(&l->w, nw * 4) == cudaSuccess && cudaMalloc(&l->grad, nw * 4) == cudaSuccess &&
              cudaMalloc(&l->bias, (size_t)out_features * 4) == cudaSuccess &&
              cudaMalloc(&l->wq, (size_t)a16(out_features) * a16(in_features)) == cudaSuccess &&
              cudaMalloc(&l->amax, sizeof(unsigned)) == cudaSuccess &&
              cudaMalloc(&l->sumsq, sizeof(double)) == cudaSuccess && cudaMalloc(&l->clip, 2 * 4) == cudaSuccess;
    ok = ok && upload(l->w, weight_f32, nw) && cudaMemset(l->grad, 0, nw * 4) == cudaSuccess;
    if (ok) {
        if (bias)
            ok = upload(l->bias, bias, (size_t)out_features);
        else
            ok = cudaMemset(l->bias, 0, (size_t)out_features * 4) == cudaSuccess;
    }
    if (!ok) {
        report_error(__FILE__, __LINE__, "trba_linear_int8_create: device allocation failed", -1);
        trba_linear_int8_destroy(l);
        return nullptr;
    }
    trba_linear_int8_requantize(l, nullptr);
    TRBA_CHECK(cudaStreamSynchronize(nullptr));
    return l;
}

void trba_linear_int8_destroy(trba_linear_int8 *l) {
    if (!l) return;
    cudaFree(l->w);
    cudaFree(l->grad);
    cudaFree(l->bias);
    cudaFree(l->wq);
    cudaFree(l->amax);
    cudaFree(l->sumsq);
    cudaFree(l->clip);
    l->a_pad.release();
    l->in_stage.release();
    l->out_stage.release();
    l->f_stage.release();
    delete l;
}

int trba_linear_int8_requantize(trba_linear_int8 *l, void *stream) {
    if (!l) return -1;
    quantize_into(l->w, l->out, l->in, l->amax, l->wq, as_stream(stream));
    return 0;
}

int trba_linear_int8_forward(trba_linear_int8 *l, const int8_t *inp, int rows, int32_t *out, void *stream) {
    TRBA_REQUIRE_RET(l && inp && out && rows > 0,
                     "LinearInt8::forward: input is not a positive multiple of in_features", -1);
    cudaStream_t st = as_stream(stream);
    if (!l->a_pad.ensure((size_t)a16(rows) * a16(l->in))) return -1;
    pad_i8(inp, l->a_pad.p, rows, l->in, st);
    launch_gemm_int8(l->a_pad.p, l->wq, out, rows, l->out, l->in, stream);
    return 0;
}

int trba_linear_int8_forward_host(trba_linear_int8 *l, const int8_t *inp, long long inp_len, int32_t *out) {
    TRBA_REQUIRE_RET(l && inp && out && inp_len > 0 && inp_len % l->in == 0,
                     "LinearInt8::forward: input is not a positive multiple of in_features", -1);
    const int rows = (int)(inp_len / l->in);
    if (!l->in_stage.ensure((size_t)inp_len) || !l->out_stage.ensure((size_t)rows * l->out)) return -1;
    if (!upload(l->in_stage.p, inp, (size_t)inp_len)) return -1;
    if (trba_linear_int8_forward(l, l->in_stage.p, rows, l->out_stage.p, nullptr)) return -1;
    TRBA_CHECK(cudaMemcpy(out, l->out_stage.p, (size_t)rows * l->out * 4, cudaMemcpyDeviceToHost));
    return 0;
}

float trba_linear_int8_backward(trba_linear_int8 *l, const float *inp, const float *grad_out, int rows, float lr,
                                float mom, void *stream) {
    (void)mom;  // unused by the reference too (src/linear.rs:121)
    if (!l || rows <= 0 || !inp || !grad_out) return 0.0f;
    cudaStream_t st = as_stream(stream);
    const float inv_rows = 1.0f / (float)rows;  // host IEEE f32 division
    const i64 nw = (i64)l->in * l->out;
    TRBA_CHECK(cudaMemsetAsync(l->sumsq, 0, sizeof(double), st));
    linear_wgrad_kernel<<<grid_for(nw), 256, 0, st>>>(inp, grad_out, rows, l->in, l->out, inv_rows, l->grad,
                                                      l->sumsq);
    TRBA_LAUNCH_CHECK();
    linear_clip_kernel<<<1, 1, 0, st>>>(l->sumsq, lr, l->clip);
    TRBA_LAUNCH_CHECK();
    linear_update_kernel<<<grid_for(nw), 256, 0, st>>>(l->w, l->grad, nw, l->clip);
    TRBA_LAUNCH_CHECK();
    linear_bias_kernel<<<grid_for(l->out), 256, 0, st>>>(l->bias, grad_out, rows, l->out, inv_rows, l->clip);
    TRBA_LAUNCH_CHECK();
    trba_linear_int8_requantize(l, stream);
    float clip = 0.0f;
    TRBA_CHECK(cudaMemcpyAsync(&clip, l->clip, 4, cudaMemcpyDeviceToHost, st));
    TRBA_CHECK(cudaStreamSynchronize(st));
    return clip;
}

float trba_linear_int8_backward_host(trba_linear_int8 *l, const float *inp, long long inp_len,
                                     const float *grad_out, long long grad_len, float lr, float mom) {
    if (!l || !inp || !grad_out) return 0.0f;
    const long long rows = inp_len / l->in;
    if (rows == 0 || grad_len < rows * l->out) return 0.0f;
    const size_t ni = (size_t)rows * l->in, ng = (size_t)rows * l->out;
    if (!l->f_stage.ensure(ni + ng)) return 0.0f;
    if (!upload(l->f_stage.p, inp, ni) || !upload(l->f_stage.p + ni, grad_out, ng)) return 0.0f;
    return trba_linear_int8_backward(l, l->f_stage.p, l->f_stage.p + ni, (int)rows, lr, mom, nullptr);
}

int trba_linear_int8_get(trba_linear_int8 *l, float *weight_f32, int8_t *weight_int8, float *bias,
                         float *grad_f32) {
    if (!l) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    const size_t nw = (size_t)l->in * l->out;
    if (weight_f32) TRBA_CHECK(cudaMemcpy(weight_f32, l->w, nw * 4, cudaMemcpyDeviceToHost));
    if (grad_f32) TRBA_CHECK(cudaMemcpy(grad_f32, l->grad, nw * 4, cudaMemcpyDeviceToHost));
    if (bias) TRBA_CHECK(cudaMemcpy(bias, l->bias, (size_t)l->out * 4, cudaMemcpyDeviceToHost));
    if (weight_int8 && !unpad_to_host(l->wq, l->out, l->in, weight_int8)) return -1;
    return 0;
}

int trba_linear_int8_set(trba_linear_int8 *l, const float *weight_f32, const float *bias) {
    if (!l) return -1;
    if (weight_f32 && !upload(l->w, weight_f32, (size_t)l->in * l->out)) return -1;
    if (bias && !upload(l->bias, bias, (size_t)l->out)) return -1;
    trba_linear_int8_requantize(l, nullptr);
    TRBA_CHECK(cudaStreamSynchronize(nullptr));
    return 0;
}

long long trba_linear_int8_param_count(const trba_linear_int8 *l) {
    return l ? (long long)l->in * l->out + l->out : -1;
}

// -------------------------------------------------------------- LSTMInt8 --
trba_lstm_int8 *trba_lstm_int8_create(int input_size, int hidden_size, const float *w_ih, const float *w_hh,
                                      const float *bias) {
    TRBA_REQUIRE_RET(input_size > 0 && hidden_size > 0 && w_ih && w_hh, "trba_lstm_int8_create: bad arguments",
                     nullptr);
    auto *l = new trba_lstm_int8;
    l->in = input_size;
    l->H = hidden_size;
    const int G = 4 * hidden_size;
    const size_t nih = (size_t)G * input_size, nhh = (size_t)G * hidden_size;
    bool ok = cudaMalloc(&l->w_ih, nih * 4) == cudaSuccess && cudaMalloc(&l->w_hh, nhh * 4) == cudaSuccess &&
              cudaMalloc(&l->bias, (size_t)G * 4) == cudaSuccess &&
              cudaMalloc(&l->q_ih, (size_t)a16(G) * a16(input_size)) == cudaSuccess &&
              cudaMalloc(&l->q_hh, (size_t)a16(G) * a16(hidden_size)) == cudaSuccess &&
              cudaMalloc(&l->amax, sizeof(unsigned)) == cudaSuccess;
    ok = ok && upload(l->w_ih, w_ih, nih) && upload(l->w_hh, w_hh, nhh);
    if (ok) {
        if (bias)
            ok = upload(l->bias, bias, (size_t)G);
        else
            ok = cudaMemset(l->bias, 0, (size_t)G * 4) == cudaSuccess;
    }
    if (!ok) {
        report_error(__FILE__, __LINE__, "trba_lstm_int8_create: device allocation failed", -1);
        trba_lstm_int8_destroy(l);
        return nullptr;
    }
    trba_lstm_int8_requantize(l, nullptr);
    TRBA_CHECK(cudaStreamSynchronize(nullptr));
    return l;
}

void trba_lstm_int8_destroy(trba_lstm_int8 *l) {
    if (!l) return;
    cudaFree(l->w_ih);
    cudaFree(l->w_hh);
    cudaFree(l->bias);
    cudaFree(l->q_ih);
    cudaFree(l->q_hh);
    cudaFree(l->amax);
    l->x_pad.release();
    l->h_pad.release();
    l->gi.release();
    l->gh.release();
    l->state.release();
    delete l;
}

int trba_lstm_int8_requantize(trba_lstm_int8 *l, void *stream) {
    if (!l) return -1;
    cudaStream_t st = as_stream(stream);
    quantize_into(l->w_ih, 4 * l->H, l->in, l->amax, l->q_ih, st);
    quantize_into(l->w_hh, 4 * l->H, l->H, l->amax, l->q_hh, st);
    return 0;
}

int trba_lstm_int8_i2h_forward(trba_lstm_int8 *l, const int8_t *x, int batch, int32_t *out, void *stream) {
    TRBA_REQUIRE_RET(l && x && out && batch > 0, "LSTMInt8::i2h_forward: bad arguments", -1);
    if (!l->x_pad.ensure((size_t)a16(batch) * a16(l->in))) return -1;
    pad_i8(x, l->x_pad.p, batch, l->in, as_stream(stream));
    launch_gemm_int8(l->x_pad.p, l->q_ih, out, batch, 4 * l->H, l->in, stream);
    return 0;
}

int trba_lstm_int8_h2h_forward(trba_lstm_int8 *l, const int8_t *h, int batch, int32_t *out, void *stream) {
    TRBA_REQUIRE_RET(l && h && out && batch > 0, "LSTMInt8::h2h_forward: bad arguments", -1);
    if (!l->h_pad.ensure((size_t)a16(batch) * a16(l->H))) return -1;
    pad_i8(h, l->h_pad.p, batch, l->H, as_stream(stream));
    launch_gemm_int8(l->h_pad.p, l->q_hh, out, batch, 4 * l->H, l->H, stream);
    return 0;
}

}  // extern "C"

namespace {

// One LSTMInt8::forward_step given the input projection gi (s32 [batch, 4H]).
bool lstm_step(trba_lstm_int8 *l, const int32_t *gi, const float *h_prev, const float *c_prev, int batch,
               float *h_new, float *c_new, float *hsum, cudaStream_t st) {
    const int H = l->H, ld = a16(H);
    if (!l->h_pad.ensure((size_t)a16(batch) * ld) || !l->gh.ensure((size_t)batch * 4 * H)) return false;
    const i64 total = (i64)a16(batch) * ld;
    quantize_h_kernel<<<grid_for(total), 256, 0, st>>>(h_prev, batch, H, ld, total, l->h_pad.p);
    TRBA_LAUNCH_CHECK();
    launch_gemm_int8(l->h_pad.p, l->q_hh, l->gh.p, batch, 4 * H, H, st);
    lstm_cell_kernel<<<grid_for((i64)batch * H), 256, 0, st>>>(gi, l->gh.p, l->bias, c_prev, batch, H, h_new, c_new,
                                                               hsum);
    TRBA_LAUNCH_CHECK();
    return true;
}

}  // namespace

extern "C" {

int trba_lstm_int8_forward_step(trba_lstm_int8 *l, const int8_t *x, const float *h_prev, const float *c_prev,
                                int batch, float *h_new, float *c_new, void *stream) {
    TRBA_REQUIRE_RET(l && x && h_prev && c_prev && h_new && c_new && batch > 0,
                     "LSTMInt8::forward_step: bad arguments", -1);
    cudaStream_t st = as_stream(stream);
    if (!l->gi.ensure((size_t)batch * 4 * l->H)) return -1;
    if (trba_lstm_int8_i2h_forward(l, x, batch, l->gi.p, stream)) return -1;
    return lstm_step(l, l->gi.p, h_prev, c_prev, batch, h_new, c_new, nullptr, st) ? 0 : -1;
}

int trba_lstm_int8_get(trba_lstm_int8 *l, float *w_ih, int8_t *w_ih_int8, float *w_hh, int8_t *w_hh_int8,
                       float *bias) {
    if (!l) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    const int G = 4 * l->H;
    if (w_ih) TRBA_CHECK(cudaMemcpy(w_ih, l->w_ih, (size_t)G * l->in * 4, cudaMemcpyDeviceToHost));
    if (w_hh) TRBA_CHECK(cudaMemcpy(w_hh, l->w_hh, (size_t)G * l->H * 4, cudaMemcpyDeviceToHost));
    if (bias) TRBA_CHECK(cudaMemcpy(bias, l->bias, (size_t)G * 4, cudaMemcpyDeviceToHost));
    if (w_ih_int8 && !unpad_to_host(l->q_ih, G, l->in, w_ih_int8)) return -1;
    if (w_hh_int8 && !unpad_to_host(l->q_hh, G, l->H, w_hh_int8)) return -1;
    return 0;
}

long long trba_lstm_int8_param_count(const trba_lstm_int8 *l) {
    return l ? 4LL * l->H * l->in + 4LL * l->H * l->H + 4LL * l->H : -1;
}

// BiLSTMInt8::forward.  The input projections of all time steps are one
// GEMM per direction (M = seq_len * batch); the recurrence then runs one
// quantise + h GEMM + cell launch per step and direction.
int trba_bilstm_int8_forward(trba_lstm_int8 *fwd, trba_lstm_int8 *bwd, const int8_t *x_seq, int batch,
                             int seq_len, float *out, void *stream) {
    TRBA_REQUIRE_RET(fwd && bwd && fwd != bwd && x_seq && out && batch > 0 && seq_len >= 0 &&
                         fwd->in == bwd->in && fwd->H == bwd->H,
                     "BiLSTMInt8::forward: bad arguments", -1);
    cudaStream_t st = as_stream(stream);
    const int H = fwd->H;
    const size_t bh = (size_t)batch * H;
    if (seq_len == 0) {
        TRBA_CHECK(cudaMemsetAsync(out, 0, bh * 2 * sizeof(float), st));
        return 0;
    }
    const int rows = seq_len * batch;
    trba_lstm_int8 *dirs[2] = {fwd, bwd};
    float *sums[2] = {nullptr, nullptr};
    for (int d = 0; d < 2; ++d) {
        trba_lstm_int8 *l = dirs[d];
        if (!l->x_pad.ensure((size_t)a16(rows) * a16(l->in)) || !l->gi.ensure((size_t)rows * 4 * H) ||
            !l->state.ensure(5 * bh))
            return -1;
        pad_i8(x_seq, l->x_pad.p, rows, l->in, st);
        launch_gemm_int8(l->x_pad.p, l->q_ih, l->gi.p, rows, 4 * H, l->in, st);
        float *h0 = l->state.p, *c0 = h0 + bh, *h1 = c0 + bh, *c1 = h1 + bh, *sum = c1 + bh;
        TRBA_CHECK(cudaMemsetAsync(l->state.p, 0, 5 * bh * sizeof(float), st));
        for (int t = 0; t < seq_len; ++t) {
            if (!lstm_step(l, l->gi.p + (size_t)t * batch * 4 * H, h0, c0, batch, h1, c1, sum, st)) return -1;
            float *th = h0, *tc = c0;
            h0 = h1;
            c0 = c1;
            h1 = th;
            c1 = tc;
        }
        sums[d] = sum;
    }
    const float inv_t = 1.0f / (float)seq_len;  // src/bilstm.rs:233
    bilstm_out_kernel<<<grid_for((i64)bh), 256, 0, st>>>(sums[0], sums[1], batch, H, inv_t, out);
    TRBA_LAUNCH_CHECK();
    return 0;
}

}  // extern "C"
