// Bandwidth-bound kernels of the drop-in ABI: BatchNorm, dynamic int8
// quantisation, SE squeeze/excite helpers, feature mean-pool and small
// utilities (src/backend.rs:111-134 of the reference's later snapshot).
//
// Numerics: every expression the reference evaluates in float is evaluated
// here with explicit round-to-nearest intrinsics in the same order, so the
// outputs match the reference's CPU backend bit for bit given the same
// inputs.  Per-channel reductions accumulate in double and round once.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------- reductions --
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum of two doubles; result valid in thread 0.
__device__ void block_sum2(double &a, double &b) {
    __shared__ double sa[32], sb[32];
    a = warp_sum(a);
    b = warp_sum(b);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    if (lane == 0) { sa[wid] = a; sb[wid] = b; }
    __syncthreads();
    if (wid == 0) {
        a = lane < nw ? sa[lane] : 0.0;
        b = lane < nw ? sb[lane] : 0.0;
        a = warp_sum(a);
        b = warp_sum(b);
    }
    __syncthreads();
}

// One CTA per channel: sum and sum of squares over [B, HW] of NCHW x, then
// mean = (float)sum / count, var = max((float)sq / count - mean^2, 0)
// (cpu_backend.cpp of the later snapshot, lines 742-768).
__global__ void bn_stats_kernel(const float *__restrict__ x, int B, int C, int HW,
                                float *__restrict__ mean, float *__restrict__ var) {
    const int c = blockIdx.x;
    double s = 0.0, q = 0.0;
    for (int b = 0; b < B; ++b) {
        const float *p = x + ((i64)b * C + c) * HW;
        for (int j = threadIdx.x; j < HW; j += blockDim.x) {
            const double v = (double)p[j];
            s += v;
            q += v * v;
        }
    }
    block_sum2(s, q);
    if (threadIdx.x == 0) {
        const float cnt = (float)((i64)B * HW);
        const float m = fdiv((float)s, cnt);
        const float v = fsub(fdiv((float)q, cnt), fmul(m, m));
        mean[c] = m;
        var[c] = v < 0.0f ? 0.0f : v;
    }
}

__device__ __forceinline__ float bn_rstd(float var, float eps) {
    return fdiv(1.0f, __fsqrt_rn(fadd(var, eps)));
}

__global__ void bn_apply_kernel(const float *__restrict__ x, const float *__restrict__ mean,
                                const float *__restrict__ var, const float *__restrict__ gamma,
                                const float *__restrict__ beta, float eps, float *__restrict__ y,
                                int C, int HW, i64 n) {
    GRID_LOOP(i, n) {
        const int c = (int)((i / HW) % C);
        const float r = bn_rstd(var[c], eps);
        y[i] = fadd(fmul(fmul(fsub(x[i], mean[c]), r), gamma[c]), beta[c]);
    }
}

// One CTA per channel: sum(dy), sum(dy * xhat) (later snapshot
// cpu_backend.cpp:782-802; the product dy*xhat is rounded to float first).
__global__ void bn_bwd_sums_kernel(const float *__restrict__ dy, const float *__restrict__ x,
                                   const float *__restrict__ mean, const float *__restrict__ var,
                                   float eps, int C, int HW, i64 n, float *__restrict__ sum_dy,
                                   float *__restrict__ sum_dy_xhat) {
    const int c = blockIdx.x;
    const float r = bn_rstd(var[c], eps), m = mean[c];
    const i64 B = n / ((i64)C * HW);
    double s = 0.0, sx = 0.0;
    for (i64 b = 0; b < B; ++b) {
        const i64 off = (b * C + c) * HW;
        for (int j = threadIdx.x; j < HW; j += blockDim.x) {
            const float d = dy[off + j];
            const float xh = fmul(fsub(x[off + j], m), r);
            s += (double)d;
            sx += (double)fmul(d, xh);
        }
    }
    block_sum2(s, sx);
    if (threadIdx.x == 0) {
        sum_dy[c] = (float)s;
        sum_dy_xhat[c] = (float)sx;
    }
}

// dx = ((gamma*r)/cnt) * ((cnt*dy - sum_dy) - xhat*sum_dy_xhat)
__global__ void bn_bwd_dx_kernel(const float *__restrict__ dy, const float *__restrict__ x,
                                 const float *__restrict__ mean, const float *__restrict__ var,
                                 const float *__restrict__ gamma, const float *__restrict__ sum_dy,
                                 const float *__restrict__ sum_dy_xhat, float eps, int C, int HW,
                                 i64 n, float cnt, float *__restrict__ dx) {
    GRID_LOOP(i, n) {
        const int c = (int)((i / HW) % C);
        const float r = bn_rstd(var[c], eps);
        const float xh = fmul(fsub(x[i], mean[c]), r);
        const float a = fdiv(fmul(gamma[c], r), cnt);
        const float t = fsub(fsub(fmul(cnt, dy[i]), sum_dy[c]), fmul(xh, sum_dy_xhat[c]));
        dx[i] = fmul(a, t);
    }
}

// max|x| into *out (zeroed by the launcher); non-negative floats order like
// their bit patterns, so an integer atomicMax is exact.
__global__ void max_abs_kernel(const float *__restrict__ x, i64 n, float *__restrict__ out) {
    float m = 0.0f;
    GRID_LOOP(i, n) m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    __shared__ float sm[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) sm[wid] = m;
    __syncthreads();
    if (wid == 0) {
        m = lane < (int)(blockDim.x >> 5) ? sm[lane] : 0.0f;
        m = warp_max(m);
        if (lane == 0) atomicMax(reinterpret_cast<int *>(out), __float_as_int(m));
    }
}

// q = rint_even(clamp(x * inv, -127, 127)), inv = 1/scale rounded on the host.
__global__ void quant_kernel(const float *__restrict__ x, i64 n, float inv, int8_t *__restrict__ q) {
    GRID_LOOP(i, n) {
        const float v = fminf(fmaxf(fmul(x[i], inv), -127.0f), 127.0f);
        q[i] = (int8_t)rint_even(v);
    }
}

__global__ void relu_quant_kernel(const float *__restrict__ y, i64 n, float inv,
                                  int8_t *__restrict__ q) {
    GRID_LOOP(i, n) {
        const float v = fminf(fmul(fmaxf(y[i], 0.0f), inv), 127.0f);
        q[i] = (int8_t)rint_even(v);
    }
}

__global__ void dequant_kernel(const int8_t *__restrict__ q, i64 n, float s, float *__restrict__ x) {
    GRID_LOOP(i, n) x[i] = fmul((float)q[i], s);
}

__global__ void add_scaled_i8_kernel(const int8_t *__restrict__ a, float sa,
                                     const int8_t *__restrict__ b, float sb, i64 n,
                                     float *__restrict__ o) {
    GRID_LOOP(i, n) o[i] = fadd(fmul((float)a[i], sa), fmul((float)b[i], sb));
}

// acc [B*Ho*Wo, ld] s32 -> out NCHW fp32 = acc * scale
__global__ void epilogue_f32_kernel(const int32_t *__restrict__ acc, int ld, float scale,
                                    float *__restrict__ out, int C, i64 hw, i64 total) {
    GRID_LOOP(i, total) {
        const i64 b = i / ((i64)C * hw);
        const int oc = (int)((i / hw) % C);
        const i64 row = b * hw + (i % hw);
        out[i] = fmul((float)acc[row * ld + oc], scale);
    }
}

// One warp per (b, c) row: mean over HW accumulated in double.
__global__ void avgpool_hw_kernel(const float *__restrict__ x, int HW, i64 rows,
                                  float *__restrict__ out) {
    const i64 warp = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const i64 nwarps = ((i64)gridDim.x * blockDim.x) >> 5;
    for (i64 r = warp; r < rows; r += nwarps) {
        double s = 0.0;
        for (int j = lane; j < HW; j += 32) s += (double)x[r * HW + j];
        s = warp_sum(s);
        if (lane == 0) out[r] = (float)(s / (double)HW);
    }
}

__global__ void avgpool_hw_bwd_kernel(const float *__restrict__ dy, int HW, i64 n,
                                      float *__restrict__ dx) {
    GRID_LOOP(i, n) dx[i] = fdiv(dy[i / HW], (float)HW);
}

__global__ void mul_gate_kernel(const float *__restrict__ x, const float *__restrict__ gate, int C,
                                int HW, i64 n, float *__restrict__ o) {
    GRID_LOOP(i, n) o[i] = fmul(x[i], gate[i / HW]);  // (b*C + c) == i / HW
}

__global__ void mask_relu_bwd_kernel(const float *__restrict__ y, const float *__restrict__ dy, i64 n,
                                     float *__restrict__ dx) {
    GRID_LOOP(i, n) dx[i] = y[i] > 0.0f ? dy[i] : 0.0f;
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, i64 n,
                           float *__restrict__ o) {
    GRID_LOOP(i, n) o[i] = fadd(a[i], b[i]);
}

__global__ void mul_kernel(const float *__restrict__ a, const float *__restrict__ b, i64 n,
                           float *__restrict__ o) {
    GRID_LOOP(i, n) o[i] = fmul(a[i], b[i]);
}

__global__ void scale_kernel(float *__restrict__ p, float s, i64 n) {
    GRID_LOOP(i, n) p[i] = fmul(p[i], s);
}

// 32x32 tiled transpose through shared memory (coalesced on both sides).
template <typename T>
__global__ void transpose_kernel(const T *__restrict__ src, int rows, int cols, T *__restrict__ dst) {
    __shared__ T tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int r = r0 + k, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[k][threadIdx.x] = src[(i64)r * cols + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int c = c0 + k, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[(i64)c * rows + r] = tile[threadIdx.x][k];
    }
}

// [B,C,H,W] -> [B,W,C], float sum over h in order, then / H.
__global__ void meanpool_h_kernel(const float *__restrict__ x, int C, int H, int W, i64 total,
                                  float *__restrict__ out) {
    GRID_LOOP(i, total) {
        const int c = (int)(i % C), w = (int)((i / C) % W);
        const i64 b = i / ((i64)C * W);
        const float *p = x + ((b * C + c) * H) * W + w;
        float s = 0.0f;
        for (int h = 0; h < H; ++h) s = fadd(s, p[(i64)h * W]);
        out[i] = fdiv(s, (float)H);
    }
}

__global__ void meanpool_h_bwd_kernel(const float *__restrict__ dy, int C, int H, int W, i64 total,
                                      float *__restrict__ dx) {
    GRID_LOOP(i, total) {
        const int c = (int)(i % C), w = (int)((i / C) % W);
        const i64 b = i / ((i64)C * W);
        const float v = fdiv(dy[i], (float)H);
        float *p = dx + ((b * C + c) * H) * W + w;
        for (int h = 0; h < H; ++h) p[(i64)h * W] = v;
    }
}

// Float -> IEEE half by mantissa truncation with denormals flushed, the
// converter of the reference's CPU mirror (cpu_backend.cpp:64-72).
__global__ void f2h_kernel(const float *__restrict__ src, uint16_t *__restrict__ dst, i64 n) {
    GRID_LOOP(i, n) {
        const uint32_t bits = __float_as_uint(src[i]);
        const uint32_t sign = (bits >> 16) & 0x8000u;
        const int32_t e = (int32_t)((bits >> 23) & 0xFFu) - 127 + 15;
        const uint32_t man = bits & 0x7FFFFFu;
        uint16_t h;
        if (e <= 0) h = (uint16_t)sign;
        else if (e >= 31) h = (uint16_t)(sign | 0x7C00u);
        else h = (uint16_t)(sign | ((uint32_t)e << 10) | (man >> 13));
        dst[i] = h;
    }
}

}  // namespace

using namespace trba;

extern "C" {

void launch_bn_stats(const float *x, int B, int C, int HW, float *mean, float *var, void *s) {
    if ((i64)B * C * HW <= 0) return;
    bn_stats_kernel<<<C, 512, 0, as_stream(s)>>>(x, B, C, HW, mean, var);
    TRBA_LAUNCH_CHECK();
}

void launch_bn_apply(const float *x, const float *mean, const float *var, const float *gamma,
                     const float *beta, float eps, float *y, int C, int HW, i64 n, void *s) {
    if (n <= 0 || C <= 0 || HW <= 0) return;
    bn_apply_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(x, mean, var, gamma, beta, eps, y, C,
                                                                HW, n);
    TRBA_LAUNCH_CHECK();
}

void launch_bn_bwd_sums(const float *dy, const float *x, const float *mean, const float *var,
                        float eps, int C, int HW, i64 n, float *sum_dy, float *sum_dy_xhat, void *s) {
    if (n <= 0 || C <= 0 || HW <= 0) return;
    bn_bwd_sums_kernel<<<C, 512, 0, as_stream(s)>>>(dy, x, mean, var, eps, C, HW, n, sum_dy,
                                                    sum_dy_xhat);
    TRBA_LAUNCH_CHECK();
}

void launch_bn_bwd_dx(const float *dy, const float *x, const float *mean, const float *var,
                      const float *gamma, const float *sum_dy, const float *sum_dy_xhat, float eps,
                      int C, int HW, i64 n, i64 count, float *dx, void *s) {
    if (n <= 0 || C <= 0 || HW <= 0) return;
    bn_bwd_dx_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(dy, x, mean, var, gamma, sum_dy,
                                                                 sum_dy_xhat, eps, C, HW, n,
                                                                 (float)count, dx);
    TRBA_LAUNCH_CHECK();
}

void launch_reduce_max_abs(const float *x, i64 n, float *out, void *s) {
    TRBA_CHECK(cudaMemsetAsync(out, 0, sizeof(float), as_stream(s)));
    if (n <= 0) return;
    max_abs_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(x, n, out);
    TRBA_LAUNCH_CHECK();
}

void launch_max_abs_f32(const float *x, float *out, i64 n, void *s) {
    launch_reduce_max_abs(x, n, out, s);
}

void launch_quant_f32_i8(const float *x, i64 n, float scale, int8_t *q, void *s) {
    if (n <= 0) return;
    const float inv = 1.0f / scale;
    quant_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(x, n, inv, q);
    TRBA_LAUNCH_CHECK();
}

void launch_relu_quant(const float *y, i64 n, float scale, int8_t *q, void *s) {
    if (n <= 0) return;
    const float inv = 1.0f / scale;
    relu_quant_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(y, n, inv, q);
    TRBA_LAUNCH_CHECK();
}

void launch_dequant_i8_f32(const int8_t *q, i64 n, float scale, float *x, void *s) {
    if (n <= 0) return;
    dequant_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(q, n, scale, x);
    TRBA_LAUNCH_CHECK();
}

void launch_add_scaled_i8(const int8_t *a, float sa, const int8_t *b, float sb, i64 n, float *out,
                          void *s) {
    if (n <= 0) return;
    add_scaled_i8_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(a, sa, b, sb, n, out);
    TRBA_LAUNCH_CHECK();
}

void launch_epilogue_f32(const int32_t *acc, int acc_ld, float scale, float *out, int C, int Ho,
                         int Wo, i64 total, void *s) {
    if (total <= 0 || C <= 0) return;
    epilogue_f32_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(acc, acc_ld, scale, out, C,
                                                                        (i64)Ho * Wo, total);
    TRBA_LAUNCH_CHECK();
}

void launch_avgpool_hw(const float *x, int C, int HW, i64 B, float *out, void *s) {
    const i64 rows = B * C;
    if (rows <= 0 || HW <= 0) return;
    avgpool_hw_kernel<<<grid_for(rows * 32), kThreads, 0, as_stream(s)>>>(x, HW, rows, out);
    TRBA_LAUNCH_CHECK();
}

void launch_avgpool_hw_backward(const float *dy, int C, int HW, i64 B, float *dx, void *s) {
    const i64 n = B * C * HW;
    if (n <= 0) return;
    avgpool_hw_bwd_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(dy, HW, n, dx);
    TRBA_LAUNCH_CHECK();
}

void launch_mul_gate(const float *x, const float *gate, int C, int HW, i64 n, float *out, void *s) {
    if (n <= 0 || HW <= 0) return;
    mul_gate_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(x, gate, C, HW, n, out);
    TRBA_LAUNCH_CHECK();
}

void launch_mask_relu_bwd(const float *y, const float *dy, i64 n, float *dx, void *s) {
    if (n <= 0) return;
    mask_relu_bwd_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(y, dy, n, dx);
    TRBA_LAUNCH_CHECK();
}

void launch_zero_f32(float *p, i64 n, void *s) {
    if (n <= 0) return;
    TRBA_CHECK(cudaMemsetAsync(p, 0, (size_t)n * sizeof(float), as_stream(s)));
}

void launch_transpose_i8(const int8_t *src, int rows, int cols, int8_t *dst, void *s) {
    if (rows <= 0 || cols <= 0) return;
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    transpose_kernel<int8_t><<<grid, block, 0, as_stream(s)>>>(src, rows, cols, dst);
    TRBA_LAUNCH_CHECK();
}

void cuda_transpose_f32(const float *src, float *dst, int rows, int cols, void *s) {
    if (rows <= 0 || cols <= 0) return;
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    transpose_kernel<float><<<grid, block, 0, as_stream(s)>>>(src, rows, cols, dst);
    TRBA_LAUNCH_CHECK();
}

void launch_add_f32(const float *a, const float *b, i64 n, float *o, void *s) {
    if (n <= 0) return;
    add_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(a, b, n, o);
    TRBA_LAUNCH_CHECK();
}

void launch_mul_f32(const float *a, const float *b, i64 n, float *o, void *s) {
    if (n <= 0) return;
    mul_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(a, b, n, o);
    TRBA_LAUNCH_CHECK();
}

void cuda_scale_vector(float *data, float scale, i64 n, void *s) {
    if (n <= 0) return;
    scale_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(data, scale, n);
    TRBA_LAUNCH_CHECK();
}

void launch_meanpool_h(const float *x, int C, int H, int W, i64 B, float *out, void *s) {
    const i64 total = B * W * C;
    if (total <= 0 || H <= 0) return;
    meanpool_h_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(x, C, H, W, total, out);
    TRBA_LAUNCH_CHECK();
}

void launch_meanpool_h_backward(const float *dy, int C, int H, int W, i64 B, float *dx, void *s) {
    const i64 total = B * W * C;
    if (total <= 0 || H <= 0) return;
    meanpool_h_bwd_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(dy, C, H, W, total, dx);
    TRBA_LAUNCH_CHECK();
}

void cuda_float_to_half(const float *src, void *dst, i64 n, void *s) {
    if (n <= 0) return;
    f2h_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(src, (uint16_t *)dst, n);
    TRBA_LAUNCH_CHECK();
}

}  // extern "C"
