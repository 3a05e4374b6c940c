// Line-image preprocessing (src/main.rs:218-239, load_image_q) for a batch
// of decoded RGB8 images: aspect-preserving resize with the triangle filter
// of the `image` crate (0.24.9, imageops::resize), white canvas, int8
// quantisation with scale 1/127.
//
// The crate resamples separably: a vertical pass into an f32 image, then a
// horizontal pass clamped to [0, 255] and rounded half away from zero.  For
// an output coordinate o over an input of length n resized to m it uses
// ratio = n / m, sratio = max(ratio, 1), the taps i in [floor(c - sratio),
// ceil(c + sratio)) clamped to the image, c = (o + 0.5) * ratio, weights
// tri((i - (c - 0.5)) / sratio) normalised by their sum, and a sequential
// f32 sum of pixel * weight.  This kernel evaluates the same expression per
// canvas pixel: one CTA per canvas row shares the row's vertical weights in
// shared memory, each thread takes canvas columns, and for every tap column
// of its horizontal window it recomputes the vertical sum in the same order
// (no intermediate image, nothing allocated).  Every operation is a single
// precision IEEE operation with round-to-nearest, written with the _rn
// intrinsics so the compiler cannot contract a multiply and an add.
#include "common.cuh"
#include "trba_preproc.h"

namespace trba {
namespace {

constexpr int kPreThreads = 256, kPreMaxTaps = 4096;

struct Window {
    int left, count;
    float ratio, sratio, centre, sum;
};

__device__ __forceinline__ float tri_w(int i, const Window &w) {
    const float x = __fdiv_rn(__fsub_rn((float)i, w.centre), w.sratio);
    const float ax = fabsf(x);
    return ax < 1.0f ? __fsub_rn(1.0f, ax) : 0.0f;
}

// Taps of output coordinate o (input length n, output length m) and the f32
// sum of their weights (summed in tap order, as the crate does).
__device__ __forceinline__ Window window(int o, int n, int m) {
    Window w;
    w.ratio = __fdiv_rn((float)n, (float)m);
    w.sratio = w.ratio < 1.0f ? 1.0f : w.ratio;
    const float support = w.sratio;  // triangle support 1 x sratio
    const float c = __fmul_rn(__fadd_rn((float)o, 0.5f), w.ratio);
    int left = (int)floorf(__fsub_rn(c, support));
    left = min(max(left, 0), n - 1);
    int right = (int)ceilf(__fadd_rn(c, support));
    right = min(max(right, left + 1), n);
    w.left = left;
    w.count = right - left;
    w.centre = __fsub_rn(c, 0.5f);
    float s = 0.0f;
    for (int i = left; i < right; ++i) s = __fadd_rn(s, tri_w(i, w));
    w.sum = s;
    return w;
}

__device__ __forceinline__ int8_t quant_px(float p) {
    const float v = __fmul_rn(__fsub_rn(__fmul_rn(__fdiv_rn(p, 255.0f), 2.0f), 1.0f), 127.0f);
    return (int8_t)fminf(fmaxf(roundf(v), -127.0f), 127.0f);
}

__global__ void __launch_bounds__(kPreThreads) preprocess_kernel(const uint8_t *__restrict__ rgb,
                                                                 const long long *__restrict__ offsets,
                                                                 const int *__restrict__ widths,
                                                                 const int *__restrict__ heights, int img_h,
                                                                 int img_w, int8_t *__restrict__ out) {
    __shared__ float vw[kPreMaxTaps];
    const int n = blockIdx.y, y = blockIdx.x;
    const int w0 = widths[n], h0 = heights[n];
    const uint8_t *src = rgb + offsets[n];
    // target size: scale = min(img_h / h0, img_w / w0) (f32), rounded, >= 1
    const float scale = fminf(__fdiv_rn((float)img_h, (float)max(h0, 1)), __fdiv_rn((float)img_w, (float)max(w0, 1)));
    const int nw = (int)fmaxf(roundf(__fmul_rn((float)w0, scale)), 1.0f);
    const int nh = (int)fmaxf(roundf(__fmul_rn((float)h0, scale)), 1.0f);
    const int y0 = img_h > nh ? (img_h - nh) / 2 : 0;
    // An image without pixels (which the reference fails to open and skips)
    // leaves a white canvas.
    const bool row_in = w0 > 0 && h0 > 0 && y >= y0 && y < y0 + nh;
    const bool copy = nw == w0 && nh == h0;
    Window vwin{};
    bool vshared = false;
    if (row_in && !copy) {
        vwin = window(y - y0, h0, nh);
        vshared = vwin.count <= kPreMaxTaps;
        if (vshared)
            for (int k = threadIdx.x; k < vwin.count; k += blockDim.x)
                vw[k] = __fdiv_rn(tri_w(vwin.left + k, vwin), vwin.sum);
    }
    __syncthreads();
    int8_t *orow = out + ((long long)n * img_h + y) * img_w * 3;
    for (int x = threadIdx.x; x < img_w; x += blockDim.x) {
        float v[3] = {255.0f, 255.0f, 255.0f};
        if (row_in && x < nw) {
            if (copy) {
                const uint8_t *p = src + ((long long)(y - y0) * w0 + x) * 3;
                v[0] = p[0], v[1] = p[1], v[2] = p[2];
            } else {
                const Window hwin = window(x, w0, nw);
                float acc[3] = {0.0f, 0.0f, 0.0f};
                for (int j = hwin.left; j < hwin.left + hwin.count; ++j) {
                    const float wj = __fdiv_rn(tri_w(j, hwin), hwin.sum);
                    float t[3] = {0.0f, 0.0f, 0.0f};
                    const uint8_t *col = src + ((long long)vwin.left * w0 + j) * 3;
                    for (int k = 0; k < vwin.count; ++k) {
                        const float wk = vshared ? vw[k] : __fdiv_rn(tri_w(vwin.left + k, vwin), vwin.sum);
                        const uint8_t *p = col + (long long)k * w0 * 3;
#pragma unroll
                        for (int c = 0; c < 3; ++c) t[c] = __fadd_rn(t[c], __fmul_rn((float)p[c], wk));
                    }
#pragma unroll
                    for (int c = 0; c < 3; ++c) acc[c] = __fadd_rn(acc[c], __fmul_rn(t[c], wj));
                }
#pragma unroll
                for (int c = 0; c < 3; ++c) v[c] = roundf(fminf(fmaxf(acc[c], 0.0f), 255.0f));
            }
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) orow[x * 3 + c] = quant_px(v[c]);
    }
}

}  // namespace
}  // namespace trba

using namespace trba;

extern "C" int trba_preprocess_lines(const uint8_t *rgb, const long long *offsets, const int *widths,
                                     const int *heights, int n, int img_h, int img_w, int8_t *out, void *stream) {
    if (n <= 0) return 0;
    if (!rgb || !offsets || !widths || !heights || !out || img_h <= 0 || img_w <= 0 || n > 65535) return -1;
    dim3 grid((unsigned)img_h, (unsigned)n);
    preprocess_kernel<<<grid, kPreThreads, 0, as_stream(stream)>>>(rgb, offsets, widths, heights, img_h, img_w, out);
    TRBA_LAUNCH_CHECK();
    return 0;
}
