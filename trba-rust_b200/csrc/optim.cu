// Device-resident conv optimiser state of the drop-in ABI (reference later
// snapshot src/backend.rs:63-104): int32 wgrad accumulation, the global
// sum of squares, Adam and Muon steps, and per-tensor weight fake-quant.
// All arithmetic follows the reference's CPU mirror exactly (f64 where it
// uses f64), so parameters match it bit for bit given the same inputs.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void grad_accum_kernel(const int32_t *__restrict__ acc, float *__restrict__ g, float scale,
                                  i64 n) {
    GRID_LOOP(i, n) g[i] = fadd(g[i], fmul((float)acc[i], scale));
}

__global__ void sum_sq_kernel(const float *__restrict__ x, i64 n, double *__restrict__ out) {
    double s = 0.0;
    GRID_LOOP(i, n) {
        const double v = (double)x[i];
        s += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double sm[32];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) atomicAdd(out, s);
    }
}

// later snapshot cpu_backend.cpp:440-456
__global__ void adam_kernel(float *__restrict__ p, const float *__restrict__ g, float *__restrict__ m,
                            float *__restrict__ v, i64 n, double lr, double wd, double clip, double b1,
                            double b2, double eps, double bc1, double bc2) {
    GRID_LOOP(i, n) {
        const double gi = __dadd_rn((double)(float)__dmul_rn((double)g[i], clip), __dmul_rn(wd, (double)p[i]));
        const float mf = (float)__dadd_rn(__dmul_rn(b1, (double)m[i]), __dmul_rn(1.0 - b1, gi));
        const float vf = (float)__dadd_rn(__dmul_rn(b2, (double)v[i]), __dmul_rn(__dmul_rn(1.0 - b2, gi), gi));
        m[i] = mf;
        v[i] = vf;
        const double mh = __ddiv_rn((double)mf, bc1), vh = __ddiv_rn((double)vf, bc2);
        const float upd = (float)__ddiv_rn(__dmul_rn(lr, mh), __dadd_rn(__dsqrt_rn(vh), eps));
        p[i] = fsub(p[i], upd);
    }
}

// later snapshot cpu_backend.cpp:1197-1213: step and decay derived from the
// device scalar gsq = ||g||_F^2.
__global__ void muon_kernel(float *__restrict__ w, const float *__restrict__ g,
                            const double *__restrict__ gsq, i64 n, double lr, double wd, double clip,
                            double min_dim, double max_dim, double cap, int autoscale) {
    const double frob = __dsqrt_rn(fmax(*gsq, 1e-30));
    const double scale = fmin(__ddiv_rn(__dsqrt_rn(min_dim), fmax(frob, 1e-8)), cap);
    const double lre = autoscale ? __dmul_rn(lr, __dsqrt_rn(max_dim)) : lr;
    const float step = (float)__dmul_rn(__dmul_rn(clip, lre), scale);
    const float dec = (float)(1.0 - __dmul_rn(lr, wd));
    GRID_LOOP(i, n) {
        const float u = fsub(fmul(w[i], dec), fmul(step, g[i]));
        w[i] = isfinite(u) ? u : 0.0f;
    }
}

// later snapshot cpu_backend.cpp:467-493: s = max/127 in f64 (1 if max == 0);
// q = roundf(clamp((float)(w / s in f64), +-127)), zero padding to [rp, kp].
__global__ void quantize_pad_kernel(const float *__restrict__ w, const float *__restrict__ max_abs,
                                    float *__restrict__ w_s_out, int8_t *__restrict__ wq, i64 rows,
                                    i64 col, i64 kp, i64 total) {
    const double mx = (double)*max_abs;
    const float s = (float)(mx > 0.0 ? __ddiv_rn(mx, 127.0) : 1.0);
    if (w_s_out && blockIdx.x == 0 && threadIdx.x == 0) *w_s_out = s;
    GRID_LOOP(i, total) {
        const i64 r = i / kp, c = i - r * kp;
        float v = 0.0f;
        if (r < rows && c < col) {
            v = (float)__ddiv_rn((double)w[r * col + c], (double)s);
            v = fminf(fmaxf(v, -127.0f), 127.0f);
        }
        wq[i] = (int8_t)roundf(v);
    }
}

}  // namespace

using namespace trba;

extern "C" {

void launch_grad_accum_i32(const int32_t *acc, float *g, float scale, i64 n, void *s) {
    if (n <= 0) return;
    grad_accum_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(acc, g, scale, n);
    TRBA_LAUNCH_CHECK();
}

void launch_sum_sq_add_f32(const float *x, double *out, i64 n, void *s) {
    if (n <= 0) return;
    sum_sq_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(x, n, out);
    TRBA_LAUNCH_CHECK();
}

void launch_adam_f32(float *p, const float *g, float *m, float *v, i64 n, double lr, double wd,
                     double clip, double b1, double b2, double eps, double bc1, double bc2, void *s) {
    if (n <= 0) return;
    adam_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(p, g, m, v, n, lr, wd, clip, b1, b2, eps,
                                                            bc1, bc2);
    TRBA_LAUNCH_CHECK();
}

void launch_muon_step_f32(float *w, const float *g, const double *gsq, i64 n, double lr, double wd,
                          double clip, double min_dim, double max_dim, double cap, i64 autoscale,
                          void *s) {
    if (n <= 0 || !w || !g || !gsq) return;
    muon_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(w, g, gsq, n, lr, wd, clip, min_dim,
                                                            max_dim, cap, autoscale ? 1 : 0);
    TRBA_LAUNCH_CHECK();
}

void launch_quantize_pad_i8(const float *w, const float *max_abs, float *w_s_out, int8_t *w_q_pad,
                            i64 rows, i64 col, i64 kp, void *s) {
    if (rows <= 0 || col <= 0) return;
    TRBA_REQUIRE(kp >= col && !(kp & 15) && w_q_pad && max_abs, "launch_quantize_pad_i8: bad args");
    const i64 rp = (rows + 15) & ~15LL, total = rp * kp;
    quantize_pad_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(w, max_abs, w_s_out, w_q_pad,
                                                                        rows, col, kp, total);
    TRBA_LAUNCH_CHECK();
}

}  // extern "C"
