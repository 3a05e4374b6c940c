// Conv helpers of the drop-in ABI: int8 im2col, the inference conv epilogue,
// the fused backward gathers (fp32 wgrad/bias, fp32 and int8-weight dgrad)
// and the 2x2 max-pools (src/backend.rs:28-60,105-110 of the reference's
// later snapshot).
//
// The dgrad gathers sum taps in the reference's order ((kh, kw) outer, output
// channel inner, one float accumulator), so their results are bit-identical
// to the reference's CPU backend; they are the operator-level entry points.
// The training step uses the tensor-core formulation in qat_model.cu.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

// One thread per byte of the padded [align16(rows), col_ld] matrix.
__global__ void im2col_pad_kernel(const int8_t *__restrict__ in, int8_t *__restrict__ col, int C,
                                  int H, int W, int kH, int kW, int sH, int sW, int pH, int pW,
                                  int Ho, int Wo, int col_ld, i64 rows, i64 total) {
    const int cols = C * kH * kW, khw = kH * kW;
    GRID_LOOP(i, total) {
        const i64 row = i / col_ld;
        const int k = (int)(i - row * col_ld);
        int8_t v = 0;
        if (row < rows && k < cols) {
            const i64 b = row / ((i64)Ho * Wo);
            const int rem = (int)(row - b * Ho * Wo);
            const int oh = rem / Wo, ow = rem - oh * Wo;
            const int ci = k / khw, kk = k - ci * khw, kh = kk / kW, kw = kk - kh * kW;
            const int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W) v = in[((b * C + ci) * H + ih) * W + iw];
        }
        col[i] = v;
    }
}

// The same operand, staged through shared memory in tiles of kTileRows = 32
// rows (output pixels).  Lane r of every warp owns row r of the tile (its
// window origin and base offset live in registers); warp w gathers input
// channels w, w + 8, ...: for a channel the kH x kW window bytes of the 32
// rows are loaded together (neighbouring lanes read neighbouring input
// pixels) and stored to the tile at column k = (c, kh, kw).  The tile is
// contiguous in col (ld = col_ld) and leaves with 16-byte stores.  KH / KW
// are compile-time for the 3x3, 2x2 and 1x1 convolutions (window bounds
// checks hoisted out of the channel loop); 0 selects run-time loops.
// Shared memory: kTileRows * (col_ld + 4) bytes (the 4-byte pad puts the 32
// rows of one column in distinct banks).
constexpr int kIm2colMaxLd = 4096;
constexpr int kTileRows = 32;

// Narrow operands (the stem convolutions: C = 3 or 16 channels, 3x3, so
// col_ld = 32 or 144 bytes): one thread per row.  The thread gathers its
// row's C * 9 window bytes (neighbouring lanes read neighbouring input
// pixels), packs them into 32-bit words in registers in K order (c, kh, kw)
// and writes the row with 16-byte stores; a warp covers 32 consecutive rows,
// i.e. one contiguous span of col.  Rows in [rows, rows_pad) are written as
// zeros.  All index arithmetic is 32-bit within an image plane.
template <int C, int KH, int KW>
__global__ void __launch_bounds__(256) im2col_rows_kernel(const int8_t *__restrict__ in, int8_t *__restrict__ col,
                                                          int H, int W, int sH, int sW, int pH, int pW, int Ho,
                                                          int Wo, i64 rows, i64 rows_pad) {
    constexpr int K = C * KH * KW, LD = (K + 15) / 16 * 16, NW = LD / 4;
    const int hwo = Ho * Wo, hw = H * W;
    for (i64 r = (i64)blockIdx.x * blockDim.x + threadIdx.x; r < rows_pad; r += (i64)gridDim.x * blockDim.x) {
        uint32_t w[NW];
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = 0u;
        if (r < rows) {
            const i64 b = r / hwo;
            const int rem = (int)(r - b * hwo), oh = rem / Wo, ow = rem - oh * Wo;
            const int ih0 = oh * sH - pH, iw0 = ow * sW - pW;
            const int8_t *src = in + b * C * hw;
            bool okh[KH], okw[KW];
#pragma unroll
            for (int i = 0; i < KH; ++i) okh[i] = (unsigned)(ih0 + i) < (unsigned)H;
#pragma unroll
            for (int j = 0; j < KW; ++j) okw[j] = (unsigned)(iw0 + j) < (unsigned)W;
#pragma unroll
            for (int c = 0; c < C; ++c)
#pragma unroll
                for (int i = 0; i < KH; ++i)
#pragma unroll
                    for (int j = 0; j < KW; ++j) {
                        const int k = (c * KH + i) * KW + j;
                        const uint32_t v =
                            (okh[i] && okw[j]) ? (uint32_t)(uint8_t)src[c * hw + (ih0 + i) * W + iw0 + j] : 0u;
                        w[k >> 2] |= v << (8 * (k & 3));
                    }
        }
        uint4 *dst = reinterpret_cast<uint4 *>(col + r * LD);
#pragma unroll
        for (int q = 0; q < NW / 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
}

// Narrow 3x3 operands with stride 1, padding 1 and W % 4 == 0 (both stem
// convolutions): one thread per four horizontally adjacent output pixels.
// For every (channel, kernel row) it reads the 32-bit word of the four input
// pixels on that input row and its two neighbour words, and forms the
// windows of kw = 0, 1, 2 with funnel shifts (window byte p = input pixel
// ow + p + kw - 1; words beyond the plane's left and right edges read as zero
// padding).  Each group of four K positions becomes one 32-bit word of each
// of the four output rows by a 4 x 4 byte transpose (byte_perm).  A warp's
// 128 output rows are one contiguous span of col: they are assembled in
// shared memory and written with 16-byte stores at consecutive addresses
// (the rows' own 16-byte pieces, written in place, sit LD * 4 bytes apart
// across the warp and measured twice as slow).  Rows in [rows, rows_pad) are
// written as zeros.  Two warps per CTA (a warp stages 128 * LD bytes).
constexpr int kQuadThreads = 64;

template <int C>
__global__ void __launch_bounds__(kQuadThreads, 12)
    im2col_quad_kernel(const int8_t *__restrict__ in, int8_t *__restrict__ col, int H, int W, i64 quads,
                       i64 quads_pad) {
    constexpr int K = C * 9, LD = (K + 15) / 16 * 16, NCH = LD / 16;
    constexpr int WB = 32 * 4 * LD;
    __shared__ __align__(16) uint8_t stage[kQuadThreads / 32][WB];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hw = H * W, plane4 = hw >> 2;
    for (i64 u0 = (i64)blockIdx.x * blockDim.x + warp * 32; u0 < quads_pad; u0 += (i64)gridDim.x * blockDim.x) {
        const i64 u = u0 + lane;
        uint8_t *sw = stage[warp] + lane * 4 * LD;
        if (u >= quads) {
#pragma unroll
            for (int p = 0; p < 4; ++p)
#pragma unroll
                for (int m = 0; m < NCH; ++m) *reinterpret_cast<uint4 *>(sw + p * LD + 16 * m) = make_uint4(0, 0, 0, 0);
        } else {
            const i64 r = 4 * u;
            const i64 b = r / hw;
            const int rem = (int)(r - b * hw), oh = rem / W, ow = rem - oh * W;
            const uint32_t *src = reinterpret_cast<const uint32_t *>(in + b * C * hw);
            const uint32_t *rowp[3];
            bool okh[3];
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
                const int ih = oh + kh - 1;
                okh[kh] = (unsigned)ih < (unsigned)H;
                rowp[kh] = src + (okh[kh] ? (ih * W + ow) >> 2 : 0);
            }
            const bool hp = ow > 0, hn = ow + 4 < W;
            auto win = [&](int k) -> uint32_t {
                if (k >= K) return 0u;
                const int c = k / 9, t = k - c * 9, kh = t / 3, kw = t - kh * 3;
                if (!okh[kh]) return 0u;
                const uint32_t *p = rowp[kh] + c * plane4;
                const uint32_t cur = p[0];
                if (kw == 1) return cur;
                if (kw == 0) return __funnelshift_r(hp ? p[-1] : 0u, cur, 24);
                return __funnelshift_r(cur, hn ? p[1] : 0u, 8);
            };
#pragma unroll
            for (int m = 0; m < NCH; ++m) {
                uint32_t rw[4][4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int k0 = 16 * m + 4 * g;
                    const uint32_t a = win(k0), bb = win(k0 + 1), cc = win(k0 + 2), d = win(k0 + 3);
                    const uint32_t t0 = __byte_perm(a, bb, 0x5140), t1 = __byte_perm(a, bb, 0x7362);
                    const uint32_t t2 = __byte_perm(cc, d, 0x5140), t3 = __byte_perm(cc, d, 0x7362);
                    rw[0][g] = __byte_perm(t0, t2, 0x5410);
                    rw[1][g] = __byte_perm(t0, t2, 0x7632);
                    rw[2][g] = __byte_perm(t1, t3, 0x5410);
                    rw[3][g] = __byte_perm(t1, t3, 0x7632);
                }
#pragma unroll
                for (int p = 0; p < 4; ++p)
                    *reinterpret_cast<uint4 *>(sw + p * LD + 16 * m) = make_uint4(rw[p][0], rw[p][1], rw[p][2], rw[p][3]);
            }
        }
        __syncwarp();
        const i64 nq = quads_pad - u0 < 32 ? quads_pad - u0 : 32;
        const int pieces = (int)(nq * 4 * LD / 16);
        uint4 *gdst = reinterpret_cast<uint4 *>(col + 4 * u0 * LD);
        for (int i = lane; i < pieces; i += 32) gdst[i] = reinterpret_cast<const uint4 *>(stage[warp])[i];
        __syncwarp();
    }
}

template <int KH, int KW>
__global__ void __launch_bounds__(256) im2col_tile_kernel(const int8_t *__restrict__ in, int8_t *__restrict__ col,
                                                          int C, int H, int W, int kH_, int kW_, int sH, int sW,
                                                          int pH, int pW, int Ho, int Wo, int col_ld, i64 rows,
                                                          i64 rows_pad) {
    extern __shared__ uint8_t tile[];
    const int kH = KH ? KH : kH_, kW = KW ? KW : kW_;
    const int pitch = col_ld + 4;
    const int khw = kH * kW, cols = C * khw;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const i64 hwo = (i64)Ho * Wo, chw = (i64)C * H * W, hw = (i64)H * W;
    const i64 ntiles = (rows_pad + kTileRows - 1) / kTileRows;
    const int chunks_per_row = col_ld >> 4;
    uint8_t *trow = tile + lane * pitch;
    for (i64 t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const i64 r0 = t * kTileRows, r = r0 + lane;
        int ih0 = -(1 << 28), iw0 = 0;  // rows past the end fail every bounds check
        i64 base = 0;
        if (r < rows) {
            const i64 b = r / hwo;
            const int rem = (int)(r - b * hwo), oh = rem / Wo, ow = rem - oh * Wo;
            ih0 = oh * sH - pH;
            iw0 = ow * sW - pW;
            base = b * chw + (i64)ih0 * W + iw0;
        }
        if constexpr (KH > 0 && KW > 0) {
            bool okh[KH], okw[KW];
#pragma unroll
            for (int i = 0; i < KH; ++i) okh[i] = (unsigned)(ih0 + i) < (unsigned)H;
#pragma unroll
            for (int j = 0; j < KW; ++j) okw[j] = (unsigned)(iw0 + j) < (unsigned)W;
            // four channels' gathers in flight per lane (the loop body's loads
            // do not depend on the previous channel's shared-memory stores)
#pragma unroll 4
            for (int c = warp; c < C; c += nwarps) {
                const int8_t *src = in + base + c * hw;
                uint8_t v[KH * KW];
#pragma unroll
                for (int i = 0; i < KH; ++i)
#pragma unroll
                    for (int j = 0; j < KW; ++j) v[i * KW + j] = (okh[i] && okw[j]) ? (uint8_t)src[i * W + j] : 0;
#pragma unroll
                for (int e = 0; e < KH * KW; ++e) trow[c * KH * KW + e] = v[e];
            }
        } else {
            for (int c = warp; c < C; c += nwarps) {
                const int8_t *src = in + base + c * hw;
                for (int i = 0; i < kH; ++i) {
                    const bool oh = (unsigned)(ih0 + i) < (unsigned)H;
                    for (int j = 0; j < kW; ++j) {
                        const bool ok = oh && (unsigned)(iw0 + j) < (unsigned)W;
                        trow[c * khw + i * kW + j] = ok ? (uint8_t)src[i * W + j] : 0;
                    }
                }
            }
        }
        for (int k = cols + warp; k < col_ld; k += nwarps) trow[k] = 0;  // K padding
        __syncthreads();
        const int live_rows = (int)min((i64)kTileRows, rows_pad - r0);
        for (int cidx = threadIdx.x; cidx < live_rows * chunks_per_row; cidx += blockDim.x) {
            const int rr = cidx / chunks_per_row, cc = cidx - rr * chunks_per_row;
            const uint32_t *srcw = reinterpret_cast<const uint32_t *>(tile + rr * pitch + cc * 16);
            *reinterpret_cast<uint4 *>(col + (r0 + rr) * col_ld + cc * 16) =
                make_uint4(srcw[0], srcw[1], srcw[2], srcw[3]);
        }
        __syncthreads();
    }
}

__global__ void im2col_f32_kernel(const int8_t *__restrict__ in, float *__restrict__ col, int C,
                                  int H, int W, int kH, int kW, int sH, int sW, int pH, int pW,
                                  int Ho, int Wo, i64 total) {
    const int cols = C * kH * kW, khw = kH * kW;
    GRID_LOOP(i, total) {
        const i64 row = i / cols;
        const int k = (int)(i - row * cols);
        const i64 b = row / ((i64)Ho * Wo);
        const int rem = (int)(row - b * Ho * Wo);
        const int oh = rem / Wo, ow = rem - oh * Wo;
        const int ci = k / khw, kk = k - ci * khw, kh = kk / kW, kw = kk - kh * kW;
        const int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
        col[i] = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                     ? (float)in[((b * C + ci) * H + ih) * W + iw]
                     : 0.0f;
    }
}

// int8 = rint_even(clamp(max(acc/div + bias, 0) * mul, -127, 127)), NCHW out.
__global__ void conv_epilogue_kernel(const int32_t *__restrict__ acc, const float *__restrict__ bias,
                                     int8_t *__restrict__ out, int ld, float div, float mul, int C,
                                     i64 hw, i64 total) {
    GRID_LOOP(i, total) {
        const i64 b = i / ((i64)C * hw);
        const int oc = (int)((i / hw) % C);
        const i64 row = b * hw + (i % hw);
        float v = fadd(fdiv((float)acc[row * ld + oc], div), bias[oc]);
        v = fmul(fmaxf(v, 0.0f), mul);
        v = fminf(fmaxf(v, -127.0f), 127.0f);
        out[i] = (int8_t)rint_even(v);
    }
}

// fp32 wgrad, one thread per weight element, direct sum in the reference's
// (b, p) order (cpu_backend.cpp:261-293).
__global__ void grad_weight_kernel(const int8_t *__restrict__ in, const float *__restrict__ go,
                                   float *__restrict__ gw, int B, int Cin, int H, int W, int Cout,
                                   int kH, int kW, int sH, int sW, int pH, int pW, int Ho, int Wo) {
    const int cols = Cin * kH * kW, hwo = Ho * Wo, khw = kH * kW;
    GRID_LOOP(i, (i64)Cout * cols) {
        const int oc = (int)(i / cols), ci = (int)(i % cols);
        const int c = ci / khw, kk = ci - c * khw, kh = kk / kW, kw = kk - kh * kW;
        float acc = 0.0f;
        for (int b = 0; b < B; ++b) {
            const int8_t *in_b = in + ((i64)b * Cin + c) * H * W;
            const float *go_b = go + ((i64)b * Cout + oc) * hwo;
            for (int p = 0; p < hwo; ++p) {
                const int oh = p / Wo, ow = p - oh * Wo;
                const int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
                if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                    acc = fadd(acc, fmul(go_b[p], (float)in_b[ih * W + iw]));
            }
        }
        gw[i] = acc;
    }
}

// Per-channel sum of go: one CTA per channel, float accumulation in the
// reference's order would serialise; a double tree sum rounds once instead.
__global__ void grad_bias_kernel(const float *__restrict__ go, float *__restrict__ gb, int B,
                                 int Cout, int hw) {
    const int oc = blockIdx.x;
    double s = 0.0;
    for (int b = 0; b < B; ++b)
        for (int j = threadIdx.x; j < hw; j += blockDim.x) s += (double)go[((i64)b * Cout + oc) * hw + j];
    __shared__ double sm[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) gb[oc] = (float)s;
    }
}

// dgrad gather, one thread per input element; W8 selects int8 weights
// (times w_scale at the end) or fp32 weights.
template <bool W8>
__global__ void grad_input_kernel(const float *__restrict__ go, const float *__restrict__ wf,
                                  const int8_t *__restrict__ wq, i64 w_ld, float w_scale,
                                  float *__restrict__ gi, int B, int Cin, int H, int W, int Cout,
                                  int kH, int kW, int sH, int sW, int pH, int pW, int Ho, int Wo) {
    const int hwo = Ho * Wo, hwi = H * W;
    GRID_LOOP(i, (i64)B * Cin * hwi) {
        const i64 bc = i / hwi;
        const int pix = (int)(i - bc * hwi);
        const int b = (int)(bc / Cin), ci = (int)(bc - (i64)b * Cin);
        const int ih = pix / W, iw = pix - ih * W;
        const float *go_b = go + (i64)b * Cout * hwo;
        float acc = 0.0f;
        for (int kh = 0; kh < kH; ++kh) {
            const int nh = ih + pH - kh;
            if (nh < 0 || nh % sH) continue;
            const int oh = nh / sH;
            if (oh >= Ho) continue;
            for (int kw = 0; kw < kW; ++kw) {
                const int nw = iw + pW - kw;
                if (nw < 0 || nw % sW) continue;
                const int ow = nw / sW;
                if (ow >= Wo) continue;
                const i64 wc = (i64)(ci * kH + kh) * kW + kw;
                const float *gp = go_b + oh * Wo + ow;
                for (int oc = 0; oc < Cout; ++oc) {
                    const float w = W8 ? (float)wq[(i64)oc * w_ld + wc] : wf[(i64)oc * w_ld + wc];
                    acc = fadd(acc, fmul(gp[(i64)oc * hwo], w));
                }
            }
        }
        gi[i] = W8 ? fmul(acc, w_scale) : acc;
    }
}

__global__ void maxpool_bwd_idx_kernel(const float *__restrict__ go, const i64 *__restrict__ idx,
                                       float *__restrict__ gi, i64 n_out, i64 n_in) {
    GRID_LOOP(i, n_out) {
        const i64 t = idx[i];
        if (t >= 0 && t < n_in) atomicAdd(gi + t, go[i]);
    }
}

// 2x2 max over int8 NCHW; ties keep the first maximum in (0,0),(0,1),(1,0),(1,1).
__global__ void maxpool_fwd_i8_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, int H,
                                      int W, i64 total) {
    const int Ho = H >> 1, Wo = W >> 1;
    GRID_LOOP(i, total) {
        const i64 bc = i / ((i64)Ho * Wo);
        const int r = (int)(i - bc * Ho * Wo), oh = r / Wo, ow = r - oh * Wo;
        const int8_t *w = x + bc * H * W + (i64)(2 * oh) * W + 2 * ow;
        int8_t m = w[0];
        if (w[1] > m) m = w[1];
        if (w[W] > m) m = w[W];
        if (w[W + 1] > m) m = w[W + 1];
        y[i] = m;
    }
}

// W % 8 == 0: one thread per four adjacent outputs.  8-byte loads of the two
// input rows, per-byte signed max of the rows and then of the horizontal
// pairs (__vmaxs4), one 4-byte store.
__global__ void maxpool_fwd_i8_v4_kernel(const int8_t *__restrict__ x, int8_t *__restrict__ y, int H, int W,
                                         i64 total4) {
    const int wq = W >> 3, Ho = H >> 1;  // output quads per output row
    GRID_LOOP(i, total4) {
        const i64 row = i / wq;  // bc * Ho + oh
        const int q = (int)(i - row * wq);
        const i64 bc = row / Ho;
        const int oh = (int)(row - bc * Ho);
        const int8_t *t = x + bc * H * W + (i64)(2 * oh) * W + 8 * q;
        const uint2 a = *reinterpret_cast<const uint2 *>(t);
        const uint2 b = *reinterpret_cast<const uint2 *>(t + W);
        const uint32_t v0 = __vmaxs4(a.x, b.x), v1 = __vmaxs4(a.y, b.y);
        const uint32_t h0 = __vmaxs4(v0, v0 >> 8), h1 = __vmaxs4(v1, v1 >> 8);
        reinterpret_cast<uint32_t *>(y)[i] = __byte_perm(h0, h1, 0x6420);
    }
}

// Backward recomputes the argmax from x; writes every element of dx.
__global__ void maxpool_bwd_i8_kernel(const int8_t *__restrict__ x, const float *__restrict__ dy,
                                      float *__restrict__ dx, int H, int W, i64 total) {
    const int Ho = H >> 1, Wo = W >> 1;
    GRID_LOOP(i, total) {
        const i64 bc = i / ((i64)Ho * Wo);
        const int r = (int)(i - bc * Ho * Wo), oh = r / Wo, ow = r - oh * Wo;
        const i64 base = bc * H * W + (i64)(2 * oh) * W + 2 * ow;
        const int8_t *w = x + base;
        int win = 0;
        int8_t m = w[0];
        if (w[1] > m) { m = w[1]; win = 1; }
        if (w[W] > m) { m = w[W]; win = 2; }
        if (w[W + 1] > m) { m = w[W + 1]; win = 3; }
        const float g = dy[i];
        dx[base] = win == 0 ? g : 0.0f;
        dx[base + 1] = win == 1 ? g : 0.0f;
        dx[base + W] = win == 2 ? g : 0.0f;
        dx[base + W + 1] = win == 3 ? g : 0.0f;
    }
}

}  // namespace

using namespace trba;

extern "C" {

void launch_im2col_pad(const int8_t *input, int8_t *col, int batch, int C, int H, int W, int kH,
                       int kW, int sH, int sW, int pH, int pW, int Ho, int Wo, int col_ld, void *s) {
    const int cols = C * kH * kW;
    const i64 rows = (i64)batch * Ho * Wo;
    if (col_ld < cols || (col_ld & 15) || rows <= 0) return;
    const i64 total = ((rows + 15) / 16 * 16) * col_ld;
    const bool aligned = (reinterpret_cast<uintptr_t>(col) & 15) == 0;
    if (aligned && kH == 3 && kW == 3 && (C == 3 || C == 16) && col_ld == (C * 9 + 15) / 16 * 16 && sH == 1 &&
        sW == 1 && pH == 1 && pW == 1 && Ho == H && Wo == W && W % 4 == 0 &&
        (reinterpret_cast<uintptr_t>(input) & 3) == 0) {
        const i64 rows_pad = (rows + 15) / 16 * 16;
        const i64 quads = rows / 4, quads_pad = rows_pad / 4;
        const unsigned grid = (unsigned)((quads_pad + kQuadThreads - 1) / kQuadThreads);
        if (C == 3)
            im2col_quad_kernel<3><<<grid, kQuadThreads, 0, as_stream(s)>>>(input, col, H, W, quads, quads_pad);
        else
            im2col_quad_kernel<16><<<grid, kQuadThreads, 0, as_stream(s)>>>(input, col, H, W, quads, quads_pad);
        TRBA_LAUNCH_CHECK();
        return;
    }
    if (aligned && kH == 3 && kW == 3 && (C == 3 || C == 16) && col_ld == (C * 9 + 15) / 16 * 16) {
        const i64 rows_pad = (rows + 15) / 16 * 16;
        const i64 want = (rows_pad + 255) / 256, cap = (i64)sm_count() * 16;
        const unsigned grid = (unsigned)(want < cap ? want : cap);
        if (C == 3)
            im2col_rows_kernel<3, 3, 3><<<grid, 256, 0, as_stream(s)>>>(input, col, H, W, sH, sW, pH, pW, Ho, Wo,
                                                                       rows, rows_pad);
        else
            im2col_rows_kernel<16, 3, 3><<<grid, 256, 0, as_stream(s)>>>(input, col, H, W, sH, sW, pH, pW, Ho, Wo,
                                                                        rows, rows_pad);
        TRBA_LAUNCH_CHECK();
        return;
    }
    if (col_ld <= kIm2colMaxLd && aligned) {
        const i64 rows_pad = (rows + 15) / 16 * 16;
        const size_t smem = (size_t)kTileRows * (col_ld + 4);
        const i64 ntiles = (rows_pad + kTileRows - 1) / kTileRows;
        const i64 cap = (i64)sm_count() * 6;  // six CTAs per SM fit (40 registers, <= 37 KB tiles)
        const unsigned grid = (unsigned)(ntiles < cap ? ntiles : cap);
        auto go = [&](auto kern) {
            static bool attr[64] = {};
            int dev = 0;
            cudaGetDevice(&dev);
            if (smem > 48 * 1024 && dev >= 0 && dev < 64 && !attr[dev]) {
                TRBA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kTileRows * (kIm2colMaxLd + 4)));
                attr[dev] = true;
            }
            kern<<<grid, kThreads, smem, as_stream(s)>>>(input, col, C, H, W, kH, kW, sH, sW, pH, pW, Ho, Wo,
                                                         col_ld, rows, rows_pad);
        };
        if (kH == 3 && kW == 3)
            go(im2col_tile_kernel<3, 3>);
        else if (kH == 2 && kW == 2)
            go(im2col_tile_kernel<2, 2>);
        else if (kH == 1 && kW == 1)
            go(im2col_tile_kernel<1, 1>);
        else
            go(im2col_tile_kernel<0, 0>);
    } else {
        im2col_pad_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(
            input, col, C, H, W, kH, kW, sH, sW, pH, pW, Ho, Wo, col_ld, rows, total);
    }
    TRBA_LAUNCH_CHECK();
}

void launch_im2col_gpu(const int8_t *input, float *col, int batch, int C, int H, int W, int kH,
                       int kW, int sH, int sW, int pH, int pW, int Ho, int Wo, void *s) {
    const i64 total = (i64)batch * Ho * Wo * C * kH * kW;
    if (total <= 0) return;
    im2col_f32_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(input, col, C, H, W, kH, kW,
                                                                      sH, sW, pH, pW, Ho, Wo, total);
    TRBA_LAUNCH_CHECK();
}

void launch_conv_epilogue(const int32_t *acc, const float *bias, int8_t *out, int acc_ld,
                          float acc_div, float out_mul, int B, int C, int Ho, int Wo, void *s) {
    const i64 hw = (i64)Ho * Wo, total = (i64)B * C * hw;
    if (total <= 0) return;
    conv_epilogue_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(acc, bias, out, acc_ld,
                                                                         acc_div, out_mul, C, hw,
                                                                         total);
    TRBA_LAUNCH_CHECK();
}

void launch_conv_backward_grad_weight(const int8_t *input, const float *go, float *gw, int B,
                                      int Cin, int H, int W, int Cout, int kH, int kW, int sH,
                                      int sW, int pH, int pW, int Ho, int Wo, void *s) {
    if (B <= 0 || Cout <= 0 || Cin <= 0) return;
    const i64 n = (i64)Cout * Cin * kH * kW;
    grad_weight_kernel<<<grid_for(n, 128), 128, 0, as_stream(s)>>>(input, go, gw, B, Cin, H, W, Cout,
                                                                   kH, kW, sH, sW, pH, pW, Ho, Wo);
    TRBA_LAUNCH_CHECK();
}

void launch_conv_backward_grad_bias(const float *go, float *gb, int B, int Cout, int Ho, int Wo,
                                    void *s) {
    if (B <= 0 || Cout <= 0) return;
    grad_bias_kernel<<<Cout, 256, 0, as_stream(s)>>>(go, gb, B, Cout, Ho * Wo);
    TRBA_LAUNCH_CHECK();
}

void launch_conv_backward_grad_input(const float *go, const float *Wt, float *gi, int B, int Cin,
                                     int H, int W, int Cout, int kH, int kW, int sH, int sW, int pH,
                                     int pW, int Ho, int Wo, void *s) {
    if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0) return;
    const i64 n = (i64)B * Cin * H * W;
    grad_input_kernel<false><<<grid_for(n), kThreads, 0, as_stream(s)>>>(
        go, Wt, nullptr, (i64)Cin * kH * kW, 1.0f, gi, B, Cin, H, W, Cout, kH, kW, sH, sW, pH, pW,
        Ho, Wo);
    TRBA_LAUNCH_CHECK();
}

void launch_conv_backward_grad_input_i8(const float *go, const int8_t *Wq, int w_ld, float w_scale,
                                        float *gi, int B, int Cin, int H, int W, int Cout, int kH,
                                        int kW, int sH, int sW, int pH, int pW, int Ho, int Wo,
                                        void *s) {
    if (B <= 0 || Cin <= 0 || H <= 0 || W <= 0) return;
    const i64 n = (i64)B * Cin * H * W;
    grad_input_kernel<true><<<grid_for(n), kThreads, 0, as_stream(s)>>>(
        go, nullptr, Wq, w_ld, w_scale, gi, B, Cin, H, W, Cout, kH, kW, sH, sW, pH, pW, Ho, Wo);
    TRBA_LAUNCH_CHECK();
}

void launch_maxpool2x2_backward(const float *go, const i64 *idx, float *gi, i64 out_n, i64 in_n,
                                void *s) {
    if (in_n > 0) TRBA_CHECK(cudaMemsetAsync(gi, 0, (size_t)in_n * sizeof(float), as_stream(s)));
    if (out_n <= 0) return;
    maxpool_bwd_idx_kernel<<<grid_for(out_n), kThreads, 0, as_stream(s)>>>(go, idx, gi, out_n, in_n);
    TRBA_LAUNCH_CHECK();
}

// Host pointers (the reference's one host-side entry, src/backend.rs:56).
void maxpool2x2_backward_host(const float *go, const uint64_t *idx, float *gi, uint64_t out_n,
                              uint64_t in_n) {
    for (uint64_t i = 0; i < in_n; ++i) gi[i] = 0.0f;
    for (uint64_t i = 0; i < out_n; ++i)
        if (idx[i] < in_n) gi[idx[i]] += go[i];
}

void launch_maxpool2x2_forward_i8(const int8_t *x, int8_t *y, int B, int C, int H, int W, void *s) {
    TRBA_REQUIRE(B > 0 && C > 0 && H >= 2 && W >= 2 && !(H & 1) && !(W & 1),
                 "launch_maxpool2x2_forward_i8: bad shape");
    const i64 total = (i64)B * C * (H / 2) * (W / 2);
    if (W % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(y) & 3) == 0) {
        maxpool_fwd_i8_v4_kernel<<<grid_for(total / 4), kThreads, 0, as_stream(s)>>>(x, y, H, W, total / 4);
    } else {
        maxpool_fwd_i8_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(x, y, H, W, total);
    }
    TRBA_LAUNCH_CHECK();
}

void launch_maxpool2x2_backward_i8(const int8_t *x, const float *dy, float *dx, int B, int C, int H,
                                   int W, void *s) {
    TRBA_REQUIRE(B > 0 && C > 0 && H >= 2 && W >= 2 && !(H & 1) && !(W & 1),
                 "launch_maxpool2x2_backward_i8: bad shape");
    const i64 total = (i64)B * C * (H / 2) * (W / 2);
    maxpool_bwd_i8_kernel<<<grid_for(total), kThreads, 0, as_stream(s)>>>(x, dy, dx, H, W, total);
    TRBA_LAUNCH_CHECK();
}

}  // extern "C"
