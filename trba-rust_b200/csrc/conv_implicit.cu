// Conv forward as an implicit GEMM on the tensor cores: the reference's
// launch_im2col_pad + launch_gemm_int8 pair (cuda/kernels.cu:476-541 and
// :227-250) without the im2col matrix.
//
// The GEMM kernel (gemm_i8.cu, ConvGather) gathers each 128-byte K slice of
// an output pixel's receptive field straight from NHWC int8 activations, so
// the operand has to be channel-innermost; this file holds the two layout
// kernels that feed it and the C entry point:
//   nhwc_from_nchw_kernel  int8 [B, C, H*W] -> [B, H*W, C] through a
//                          shared-memory tile of 64 pixels x 128 channels;
//   wh_from_wq_kernel      int8 weights from the reference's K order
//                          (ci, ky, kx) to the gather's (ky, kx, ci).
#include <mutex>

#include "common.cuh"
#include "conv_implicit.cuh"
#include "gemm_i8.cuh"
#include "trba_b200.h"
#include "trba_backend.h"

namespace trba {
namespace {

constexpr int kTpPix = 64;        // pixels per tile
constexpr int kTpChan = 128;      // channels per tile
constexpr int kTpStride = kTpPix + 1;  // shared-memory row stride (bytes): spreads a column over the banks

// Grid (ceil(HW / 64), ceil(C / 128), B), 256 threads.
__global__ void __launch_bounds__(256) nhwc_from_nchw_kernel(const int8_t *__restrict__ in, int8_t *__restrict__ out,
                                                             int C, int HW) {
    __shared__ uint8_t tile[kTpChan * kTpStride];
    const int p0 = blockIdx.x * kTpPix, c0 = blockIdx.y * kTpChan, b = blockIdx.z;
    const int np = min(kTpPix, HW - p0), nc = min(kTpChan, C - c0);
    const int8_t *src = in + ((i64)b * C + c0) * HW + p0;
    // load: 16 threads per channel row, four pixels each
    const bool vec = (HW & 3) == 0 && (reinterpret_cast<uintptr_t>(in) & 3) == 0;
    for (int i = threadIdx.x; i < nc * 16; i += blockDim.x) {
        const int c = i >> 4, p = (i & 15) * 4;
        uint8_t *t = tile + c * kTpStride + p;
        const int8_t *s = src + (i64)c * HW + p;
        if (vec && p + 4 <= np) {
            const char4 v = *reinterpret_cast<const char4 *>(s);
            t[0] = (uint8_t)v.x, t[1] = (uint8_t)v.y, t[2] = (uint8_t)v.z, t[3] = (uint8_t)v.w;
        } else {
            for (int j = 0; j < 4 && p + j < np; ++j) t[j] = (uint8_t)s[j];
        }
    }
    __syncthreads();
    // store: one thread per (pixel, 16 channels), channel groups fastest, so a
    // warp writes whole contiguous pixel rows
    const int groups = nc >> 4;  // C is a multiple of 16
    int8_t *dst = out + ((i64)b * HW + p0) * C + c0;
    for (int i = threadIdx.x; i < np * groups; i += blockDim.x) {
        const int p = i / groups, g = i - p * groups;
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint8_t *t = tile + (16 * g + 4 * k) * kTpStride + p;
            w[k] = (uint32_t)t[0] | ((uint32_t)t[kTpStride] << 8) | ((uint32_t)t[2 * kTpStride] << 16) |
                   ((uint32_t)t[3 * kTpStride] << 24);
        }
        *reinterpret_cast<uint4 *>(dst + (i64)p * C + 16 * g) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// wh[n, (ky*kw + kx)*cin + ci] = wq[n, ci*kh*kw + ky*kw + kx], n < cout.
__global__ void wh_from_wq_kernel(const int8_t *__restrict__ wq, int w_ld, int8_t *__restrict__ wh, int cout, int cin,
                                  int khw) {
    const i64 K = (i64)cin * khw, n_el = (i64)cout * K;
    for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < n_el; e += (i64)gridDim.x * blockDim.x) {
        const int n = (int)(e / K), k = (int)(e - (i64)n * K);
        const int tap = k / cin, ci = k - tap * cin;
        wh[e] = wq[(i64)n * w_ld + (i64)ci * khw + tap];
    }
}

std::mutex g_scr_mu;
uint8_t *g_scr[64] = {};
size_t g_scr_bytes[64] = {};

}  // namespace

void nhwc_from_nchw_i8(const int8_t *in, int8_t *out, int B, int C, int HW, cudaStream_t st) {
    if (B <= 0 || C <= 0 || HW <= 0) return;
    const dim3 grid((unsigned)((HW + kTpPix - 1) / kTpPix), (unsigned)((C + kTpChan - 1) / kTpChan), (unsigned)B);
    nhwc_from_nchw_kernel<<<grid, 256, 0, st>>>(in, out, C, HW);
    TRBA_LAUNCH_CHECK();
}

}  // namespace trba

extern "C" int trba_conv_gemm_int8_implicit(const int8_t *input, const int8_t *weight_q, int w_ld, int32_t *acc, int b,
                                            int cin, int h, int w, int cout, int kh, int kw, int sh, int sw, int ph,
                                            int pw, int ho, int wo, void *stream) {
    using namespace trba;
    if (b <= 0 || cin <= 0 || h <= 0 || w <= 0 || cout <= 0 || ho <= 0 || wo <= 0) return 0;
    const bool pow2 = cin >= 16 && cin <= 1024 && (cin & (cin - 1)) == 0;
    if (!pow2 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || ph < 0 || pw < 0 || w_ld < cin * kh * kw ||
        ho != (h + 2 * ph - kh) / sh + 1 || wo != (w + 2 * pw - kw) / sw + 1) {
        report_error(__FILE__, __LINE__,
                     "trba_conv_gemm_int8_implicit: unsupported conv (cin a power of two in [16, 1024], w_ld >= "
                     "cin*kh*kw, ho/wo the conv's output size)", -1);
        return -1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return e != cudaSuccess ? (int)e : -1;
    const int K = cin * kh * kw;
    const size_t x_bytes = ((size_t)b * h * w * cin + 255) & ~size_t(255);
    const size_t need = x_bytes + (size_t)cout * K;
    uint8_t *buf = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scr_mu);
        if (g_scr_bytes[dev] < need) {
            if (g_scr[dev]) TRBA_CHECK(cudaFree(g_scr[dev]));
            g_scr[dev] = nullptr;
            g_scr_bytes[dev] = 0;
            e = cudaMalloc(&g_scr[dev], need);
            if (e != cudaSuccess) {
                report_error(__FILE__, __LINE__, "trba_conv_gemm_int8_implicit: scratch allocation", (int)e);
                return (int)e;
            }
            g_scr_bytes[dev] = need;
        }
        buf = g_scr[dev];
    }
    cudaStream_t st = as_stream(stream);
    int8_t *xh = reinterpret_cast<int8_t *>(buf), *wh = reinterpret_cast<int8_t *>(buf + x_bytes);
    const int before = trba_last_error();
    nhwc_from_nchw_i8(input, xh, b, cin, h * w, st);
    wh_from_wq_kernel<<<grid_for((i64)cout * K), 256, 0, st>>>(weight_q, w_ld, wh, cout, cin, kh * kw);
    TRBA_LAUNCH_CHECK();
    const ConvGeo g{xh, b, h, w, cin, kh, kw, sh, sw, ph, pw, ho, wo};
    if (!gemm_i8_conv_implicit_s32(g, wh, K, cout, acc, st)) {
        report_error(__FILE__, __LINE__, "trba_conv_gemm_int8_implicit: operands not TMA-describable", -1);
        return -1;
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    const int after = trba_last_error();
    return after != before ? (after ? after : -1) : 0;
}
