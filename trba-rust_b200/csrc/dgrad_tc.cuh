// Conv input gradient on the tensor cores (tcgen05 kind::f16), as an
// implicit GEMM over stride-phase classes.
//
//   gi[b, ci, y, x] = w_s * sum_{(kh, kw), co} dy[b, co, oy, ox] * Wq[co, ci, kh, kw]
//   with oy = (y + pH - kh) / sH, ox = (x + pW - kw) / sW on the output grid
//
// (the reference's launch_conv_backward_grad_input_i8, later snapshot
// cuda/kernels.cu:913-957, and src/qnet.rs:1068-1080).
//
// Input pixels are split into classes by their stride phase (y mod sH,
// x mod sW): within a class every pixel uses the same set of kernel taps, so
// the class is a dense GEMM with M = its pixels, N = Cin and K = taps x Cout
// (no zero taps in the operand, only the plane border).  The int8 weights
// are exact in bf16; the fp32 dy is written as the sum of three bf16 terms
// (hi + mid + lo carry its 24-bit significand), and the three products are
// accumulated into one fp32 TMEM accumulator.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace trba {
namespace dgtc {

constexpr int kMaxClasses = 4;
constexpr int kMaxTaps = 16;
constexpr int kChunk = 64;  // K values per shared-memory stage row (128 bytes of bf16)

struct Class {
    int py, px;    // stride phase of the class's input pixels
    int Hc, Wc;    // class sub-grid (pixels y = py + sH * i, x = px + sW * j)
    int ntaps;     // kernel taps that reach the output grid from this phase
    int kchunks;   // ceil(ntaps * Cout / 64): K chunks of the class GEMM
    int b_off;     // first chunk (halo tiling: first weight block) of this class in the weight image
    int tile0;     // first tile of this class in the launch (batch dependent)
    int mtiles;    // M tiles of this class (batch dependent)
    int8_t kh[kMaxTaps], kw[kMaxTaps];
};

// The halo tiling (Cout a multiple of 16): the three dy planes hold dy on a
// padded grid of Hq x Wq positions per image (real values at rows < Ho and
// columns < Wo of each image's slot, zeros in the gap rows and columns,
// which the neighbouring image and row share).  Class pixel (i, j) of a
// stride phase (y = py + sH i, x = px + sW j) reads dy at (i + dh, j + dw)
// for each of its taps, dh = (py + pH - kh) / sH (exact within the class),
// so on the padded grid the rows a tap reads for a run of consecutive
// positions (b, i, j) are that run shifted by the tap's offset dh * Wq + dw:
// every class is a stride-1 problem over the same planes.  A tile is 128 * mb
// consecutive positions of one class; one copy of its halo (128 * mb +
// dmax - dmin rows) per KC output channels serves every tap of the class.
// Positions outside the class grid are computed and not stored.
struct Halo {
    int Hq, Wq;         // padded slot of one image
    int mb;             // 128-row MMA blocks per tile (the tile has 128 * mb positions)
    int KC;             // output channels (K) per halo stage: 16, 32 or 64
    int nchunks;        // Cout / KC
    int dmin, dmax;     // smallest (<= 0) and largest (>= 0) tap offset over all classes
    int R;              // halo rows per tile
    int sa, sb;         // shared-memory stages of halos and of weight blocks
    int nacc;           // TMEM accumulators (2: double-buffered, 1 when 2 x mb x BN columns do not fit)
    int taps;           // taps of all classes (weight blocks per N tile and chunk)
    int off[kMaxClasses][kMaxTaps];  // tap offset from the halo's first row
    long long mpos;     // B * Hq * Wq (batch dependent)
    long long rows;     // rows of one plane slab, guards included (batch dependent)
};

struct Plan {
    int ncls;
    int Cin, Cout, H, W, Ho, Wo, kH, kW, sH, sW, pH, pW;
    int lgCout, lgSH, lgSW;  // log2 of Cout and of the strides (all powers of two)
    int Npad;          // Cin rounded up to the N tile
    int BN;            // N of one MMA tile: 16, 32, 64 or 128
    int ntn;           // N tiles (Npad / BN)
    int total_chunks;  // chunks of the weight image (sum over classes)
    int B;             // batch of the launch
    int tiles;         // tiles of the launch (batch dependent)
    Class cls[kMaxClasses];
    int halo;  // 1: halo tiling
    Halo h;
};

// Builds the plan of a conv, or returns false when the kernel does not
// serve it (Cout or a stride not a power of two, Cout < 8, more than 4
// stride phases or 16 taps per phase).  Stride-1 convs with Cout a multiple
// of 16 and padding below the kernel size get the halo tiling, as do
// strided convs whose phase classes fit it.
// Batch-dependent fields are filled by set_batch.
bool make_plan(int Cin, int Cout, int H, int W, int kH, int kW, int sH, int sW, int pH, int pW, int Ho, int Wo,
               Plan &p);
void set_batch(Plan &p, int B);
// Tiling override for tests and tuning (process wide, read by make_plan):
// mb < 0 keeps every conv on the class tiling; mb == 0 chooses the halo
// tile by the cost model; mb in 1..4 forces 128 * mb positions per tile
// and, when kc is 16, 32 or 64, KC output channels per halo stage.
void set_tiling_override(int mb, int kc);
// Elements (bf16) of the weight image of a plan.
__host__ __device__ inline long long image_elements(const Plan &p) {
    return p.halo ? (long long)p.Npad * p.Cout * p.h.taps : (long long)p.total_chunks * p.Npad * kChunk;
}
// Bytes of the bf16 weight image of a plan.
inline long long weight_image_bytes(const Plan &p) { return 2 * image_elements(p); }

// Device-side writer of the weight image: element (chunk gc, row n, k of
// the chunk) of the image of `p` holds bf16(wq[co, n, kh, kw]) for the tap
// and output channel that k selects, zero past the taps or past Cin; stored
// in the 128-byte-swizzled K-major layout the MMA reads, so one bulk copy
// of `BN` rows places a stage's operand.  wq: [a16(Cout), kp] int8 with K
// order (ci, kh, kw) (the forward GEMM operand).
__device__ __forceinline__ void image_entry(const Plan &p, long long e, int &gc, int &n, int &kl) {
    kl = (int)(e & 63);
    const long long r = e >> 6;
    n = (int)(r % p.Npad);
    gc = (int)(r / p.Npad);
}
__device__ __forceinline__ long long image_offset(int gc, int n, int kl, int Npad) {
    return ((long long)gc * Npad + n) * 128 + ((((kl >> 3) ^ (n & 7))) << 4) + (kl & 7) * 2;
}
// Source K index (ci * kh*kw + tap) in the forward operand of image element
// (gc, n, kl), or -1 for a zero entry.
__device__ __forceinline__ int image_source(const Plan &p, int gc, int n, int kl, int &co) {
    int c = 0;
    while (c + 1 < p.ncls && gc >= p.cls[c + 1].b_off) ++c;
    const Class &C = p.cls[c];
    const int k = (gc - C.b_off) * kChunk + kl;
    const int tap = k / p.Cout;
    co = k - tap * p.Cout;
    if (tap >= C.ntaps || n >= p.Cin) return -1;
    return n * p.kH * p.kW + C.kh[tap] * p.kW + C.kw[tap];
}

// Element e (0 <= e < image_elements) of the weight image of either tiling:
// its byte offset in the image (*dst), its output channel (*co) and its
// source K index in the forward operand, or -1 for a zero entry.  The halo
// image is blocks of [KC / 8][BN rows][8] bf16, one per (class, N tile,
// channel chunk, tap of the class) in that order (class c's first block is
// cls[c].b_off): the no-swizzle K-major layout one bulk copy places as a
// weight stage.
__device__ __forceinline__ int image_element(const Plan &p, long long e, int &co, long long &dst) {
    if (!p.halo) {
        int gc, n, kl;
        image_entry(p, e, gc, n, kl);
        dst = image_offset(gc, n, kl, p.Npad);
        return image_source(p, gc, n, kl, co);
    }
    dst = 2 * e;
    const int j = (int)(e & 7);
    long long q = e >> 3;
    const int r = (int)(q % p.BN);
    q /= p.BN;
    const int nsl = p.h.KC >> 3;
    const int s = (int)(q % nsl);
    q /= nsl;  // weight block
    int k = 0;
    while (k + 1 < p.ncls && q >= p.cls[k + 1].b_off) ++k;
    const Class &C = p.cls[k];
    q -= C.b_off;
    const int t = (int)(q % C.ntaps);
    q /= C.ntaps;
    const int c = (int)(q % p.h.nchunks);
    const int nt = (int)(q / p.h.nchunks);
    co = c * p.h.KC + s * 8 + j;
    const int ci = nt * p.BN + r;
    return ci < p.Cin ? ci * p.kH * p.kW + C.kh[t] * p.kW + C.kw[t] : -1;
}

// Elements of one bf16 plane of dy: NHWC, B x Ho x Wo x Cout for the class
// tiling; [Cout / 8][h.rows][8] for the halo tiling.  The launch needs a
// scratch of 3 planes.
inline long long plane_elements(const Plan &p) {
    return p.halo ? (long long)p.Cout * p.h.rows : (long long)p.B * p.Ho * p.Wo * p.Cout;
}

// gi (NCHW f32) from dy (NCHW f32) and the weight image: two launches (the
// split of dy into three bf16 planes, in `planes`, then the tensor-core
// GEMM).  ws_co (optional, per-output-channel weight scales): dy[b, co] is
// multiplied by ws_co[co] before the split.  Epilogue as the exact
// kernel's: v = acc * w_s (the device scalar w_s, or w_s_val when w_s is
// null); v = mask_q[i] > 0 ? v : 0 (when mask_q); v += add[i] (when add);
// gi[i] = v; and, when gmax_out, atomic max of |v * gmax_scale| into
// gmax_out.  add may alias gi.
void launch(const Plan &p, const uint8_t *wimg, uint16_t *planes, const float *dy, const float *w_s, float w_s_val,
            const float *ws_co, const int8_t *mask_q, const float *add, float *gi, const float *gmax_scale,
            float *gmax_out, cudaStream_t st);

// Writes the weight image of `p` from an int8 weight matrix [Cout rows,
// w_ld] with K order (ci, kh, kw).
__global__ void image_from_wq_kernel(const __grid_constant__ Plan P, const int8_t *__restrict__ wq, int w_ld,
                                     uint8_t *__restrict__ wimg);

// Device error word of this kernel (a bounded wait gave up); clears it when
// clear.  Synchronises the device.
int error_poll(bool clear);

}  // namespace dgtc
}  // namespace trba
