// Conv input gradient on the tensor cores: implicit GEMM per stride-phase
// class, tcgen05.mma kind::f16 with bf16 operands and an fp32 TMEM
// accumulator (the plan and the operand contract are in dgrad_tc.cuh).
//
// Two launches per input gradient:
//   split_nhwc_kernel   dy (NCHW f32, optionally times a per-output-channel
//                       weight scale) -> three bf16 planes hi / mid / lo in
//                       NHWC order, so that the 64 values of one K chunk of
//                       one pixel (one tap, 64 output channels) are 128
//                       contiguous bytes of each plane.  The split is exact:
//                       hi = v with the low 16 significand bits cleared,
//                       mid = (v - hi) likewise, lo = v - hi - mid; each
//                       subtraction is exact and lo has at most 8 significant
//                       bits, so hi + mid + lo == v and every product with an
//                       int8 weight is exact in fp32.  The only rounding is
//                       the tensor core's fp32 accumulation.
//   dgrad_tc_kernel     one CTA per SM, persistent over 128-pixel tiles,
//                       9 warps:
//     warps 0..3  producers: 16-byte cp.async copies of the three planes'
//                 rows of the tile's pixels at the chunk's tap into the
//                 A operands of a shared-memory stage (128-byte rows,
//                 16-byte pieces XOR-swizzled by row, the layout TMA's
//                 SWIZZLE_128B produces; zero-filled where the tap leaves
//                 the output grid); each thread's copies of a stage arrive
//                 on the stage's barrier when they land, so producers run
//                 ahead over every free stage; thread 0 bulk-copies the
//                 stage's weight chunk, pre-swizzled in global memory.
//     warp 4      MMA issuer (lane 0): per stage, 3 terms x 4 MMAs of
//                 M = 128, N = BN, K = 16 into one of two TMEM
//                 accumulators, so the epilogue of a tile overlaps the MMAs
//                 of the next.
//     warps 5..8  epilogue: tcgen05.ld of the accumulator (one pixel row
//                 per thread), times w_s, STE mask, residual add, NCHW
//                 store and the max |gi * scale| of the next
//                 re-quantisation.
//
// Every mbarrier wait is bounded (2 s): on a timeout the CTA raises an
// abort flag, every role leaves its loop, issued weight copies are drained,
// TMEM is freed and g_dgtc_error is set for the host to read.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "dgrad_tc.cuh"
#include "tc_primitives.cuh"
#include "trba_b200.h"
#include "trba_backend.h"

using namespace trba;
using namespace trba::tc;

namespace trba {
namespace dgtc {

__device__ int g_dgtc_error = 0;

namespace {

constexpr int kRows = 128;                      // UMMA M: pixels per tile
constexpr int kRowBytes = 128;                  // 64 bf16 of K per stage row
constexpr int kPartBytes = kRows * kRowBytes;   // one split term of A: 16 KB
constexpr int kProdWarps = 4;                   // one A row per producer thread
constexpr int kMmaWarp = kProdWarps;
constexpr int kEpiWarps = 4;                    // one per TMEM lane quarter
constexpr int kThreads = 32 * (kProdWarps + 1 + kEpiWarps);
constexpr int kMaxStages = 4;
constexpr size_t kSmemBudget = 224 * 1024;

struct Ctl {
    uint64_t afull[kMaxStages];  // producer arrivals (128)
    uint64_t bfull[kMaxStages];  // weight chunk bulk copy (transaction bytes)
    uint64_t empty[kMaxStages];  // MMA commit: the stage may be refilled
    uint64_t tfull[2];           // accumulator ready for the epilogue
    uint64_t tempty[2];          // accumulator drained (one arrival per epilogue warp)
    uint64_t drained;
    uint32_t tmem_base;
    int abort;
    uint32_t b_issued, b_consumed;
};

struct Args {
    const uint16_t *planes;  // hi, mid, lo bf16 planes of dy, NHWC, plane_elems apart
    long long plane_elems;
    const uint8_t *wimg;
    const float *w_s;  // device scalar, or null: w_s_val
    float w_s_val;
    const int8_t *mask_q;
    const float *add;
    float *gi;
    const float *gmax_scale;
    float *gmax_out;
    int B;
    int stages;
    unsigned long long wait_ns;  // limit of every pipeline wait
    int skip_weights;            // self-test: never issue the weight copies (the waits give up)
};

__device__ __forceinline__ int tile_class(const Plan &P, int t) {
    int c = 0;
    while (c + 1 < P.ncls && t >= P.cls[c + 1].tile0) ++c;
    return c;
}

// Pixel of row m of a class (m < B * Hc * Wc): image b, input row y, column x.
__device__ __forceinline__ void class_pixel(const Plan &P, const Class &C, int m, int &b, int &y, int &x) {
    const int hw = C.Hc * C.Wc;
    b = m / hw;
    const int q = m - b * hw;
    const int yy = q / C.Wc;
    y = C.py + P.sH * yy;
    x = C.px + P.sW * (q - yy * C.Wc);
}

// Three bf16 terms of a pair of floats, packed (element 0 in the low half).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &mid, uint32_t &lo) {
    const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    const float ha = __uint_as_float(ua & 0xffff0000u), hb = __uint_as_float(ub & 0xffff0000u);
    const float ra = __fsub_rn(a, ha), rb = __fsub_rn(b, hb);
    const uint32_t ura = __float_as_uint(ra), urb = __float_as_uint(rb);
    const float ma = __uint_as_float(ura & 0xffff0000u), mb = __uint_as_float(urb & 0xffff0000u);
    const float la = __fsub_rn(ra, ma), lb = __fsub_rn(rb, mb);
    hi = __byte_perm(ua, ub, 0x7632);
    mid = __byte_perm(ura, urb, 0x7632);
    lo = __byte_perm(__float_as_uint(la), __float_as_uint(lb), 0x7632);
}

template <int BN>
struct Geo {
    static constexpr int B_BYTES = BN * kRowBytes;
    static constexpr int STAGE = 3 * kPartBytes + B_BYTES;  // multiple of 1024
    static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int CW = 16;  // accumulator columns per tcgen05.ld (BN >= 16)
};

template <int CW>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[CW]) {
    if constexpr (CW == 16) tmem_ld_32x32b_x16(taddr, v);
    else tmem_ld_32x32b_x32(taddr, v);
}

// Epilogue of CW accumulator columns of one output pixel (row of the tile):
// every STE-mask and residual value of the columns is loaded first, so the
// loads are in flight together (`add` may alias `gi`, but each element is
// read before it is written), then the values are scaled, masked, added and
// stored, and |v * gsc| goes into the running max.  Columns j < nvalid are
// real input channels; rv: the row is a real pixel; base: its element of
// column 0 (NCHW, channel stride HW).
template <int CW>
__device__ __forceinline__ void epilogue_cols(const uint32_t (&v)[CW], bool any, float ws, const Args &a, i64 base,
                                              int HW, int nvalid, bool rv, float gsc, float &gm) {
    // 16 columns per batch, addressed by 32-bit offsets from the row's base
    // pointers (CW planes of one image fit an int offset)
    float *gi = a.gi + base;
    const float *add = a.add ? a.add + base : nullptr;
    const int8_t *mq = a.mask_q ? a.mask_q + base : nullptr;
#pragma unroll
    for (int h = 0; h < CW; h += 16) {
        constexpr int NB = CW < 16 ? CW : 16;
        float av[NB];
        bool keep[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const bool ok = rv && h + j < nvalid;
            const int o = (h + j) * HW;
            av[j] = (ok && add) ? add[o] : 0.0f;
            keep[j] = (ok && mq) ? mq[o] > 0 : true;
        }
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            if (rv && h + j < nvalid) {
                float val = any ? fmul(__uint_as_float(v[h + j]), ws) : 0.0f;
                if (mq) val = keep[j] ? val : 0.0f;
                if (add) val = fadd(val, av[j]);
                gi[(h + j) * HW] = val;
                gm = fmaxf(gm, fabsf(fmul(val, gsc)));
            }
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) dgrad_tc_kernel(const __grid_constant__ Plan P, const Args a) {
    using G = Geo<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int stages = a.stages;
    Ctl *ctl = reinterpret_cast<Ctl *>(smem + (size_t)stages * G::STAGE);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&ctl->afull[s], kProdWarps * 32);
            mbar_init(&ctl->bfull[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&ctl->tfull[i], 1);
            mbar_init(&ctl->tempty[i], kEpiWarps);
        }
        mbar_init(&ctl->drained, 1);
        ctl->abort = 0;
        ctl->b_issued = 0;
        ctl->b_consumed = 0;
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&ctl->tmem_base, G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ctl->tmem_base;
    volatile int *abort = &ctl->abort;
    const int HoWo = P.Ho * P.Wo;

    if (warp < kProdWarps) {
        // ------------------------------------------------ producers
        // Thread (rs, l8): 16-byte piece l8 of the 128-byte rows rs + 16 i
        // (i < 8) of every A operand; the piece's 8 K values belong to one
        // tap (Cout is a power of two >= 8).
        const int l8 = threadIdx.x & 7, rs = threadIdx.x >> 3;
        const int lgC = P.lgCout;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < P.tiles && !*abort; t += gridDim.x) {
            const Class &C = P.cls[tile_class(P, t)];
            if (C.kchunks == 0) continue;  // a phase without taps: the epilogue alone writes it
            const int local = t - C.tile0, mt = local / P.ntn, n0 = (local - mt * P.ntn) * BN;
            int py[8], px[8], pb[8];  // rows' pixels: input row, column, b * Ho * Wo (-1: past the end)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int m = mt * kRows + rs + 16 * i;
                int b = 0, y = 0, x = 0;
                const bool rv = m < a.B * C.Hc * C.Wc;
                if (rv) class_pixel(P, C, m, b, y, x);
                py[i] = y, px[i] = x, pb[i] = rv ? b * HoWo : -1;
            }
            for (int kc = 0; kc < C.kchunks; ++kc, ++it) {
                const int s = it % stages;
                const uint32_t ph = (it / stages) & 1u;
                if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort, a.wait_ns)) break;
                uint8_t *stage = smem + (size_t)s * G::STAGE;
                if (threadIdx.x == 0 && !a.skip_weights) {
                    mbar_expect_tx(&ctl->bfull[s], G::B_BYTES);
                    bulk_load(stage + 3 * kPartBytes, a.wimg + ((i64)(C.b_off + kc) * P.Npad + n0) * kRowBytes,
                              G::B_BYTES, &ctl->bfull[s]);
                    ctl->b_issued = it + 1;
                }
                const int k0 = kc * kChunk + l8 * 8;
                const int tap = k0 >> lgC, co = k0 & (P.Cout - 1);
                const bool tok = tap < C.ntaps;
                const int dh = tok ? P.pH - C.kh[tap] : 0, dw = tok ? P.pW - C.kw[tap] : 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int r = rs + 16 * i;
                    const int ny = py[i] + dh, nx = px[i] + dw;
                    const int oy = ny >> P.lgSH, ox = nx >> P.lgSW;  // exact: the class fixes the phase
                    const bool ok = tok && pb[i] >= 0 && ny >= 0 && nx >= 0 && oy < P.Ho && ox < P.Wo;
                    const i64 e = ok ? ((i64)(pb[i] + oy * P.Wo + ox) << lgC) + co : 0;
                    uint8_t *dst = stage + r * kRowBytes + ((l8 ^ (r & 7)) << 4);
#pragma unroll
                    for (int p = 0; p < 3; ++p)
                        cp_async16(dst + p * kPartBytes, a.planes + p * a.plane_elems + e, ok ? 16u : 0u);
                }
                // the stage's barrier receives this thread's arrival when its
                // copies have landed: no waiting here, the next chunk's copies
                // go out at once (the MMA warp fences the async proxy)
                cp_async_arrive_noinc(&ctl->afull[s]);
            }
        }
        cp_async_wait<0>();  // nothing may land after the CTA is gone
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(kRows, BN);
            uint32_t it = 0, acc = 0, acc_ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < P.tiles && ok; t += gridDim.x) {
                const Class &C = P.cls[tile_class(P, t)];
                if (!(ok = mbar_wait(&ctl->tempty[acc], acc_ph ^ 1u, abort, a.wait_ns))) break;
                tc_fence_after();
                const uint32_t d = tbase + acc * BN;
                for (int kc = 0; kc < C.kchunks; ++kc, ++it) {
                    const int s = it % stages;
                    const uint32_t ph = (it / stages) & 1u;
                    if (!(ok = mbar_wait(&ctl->bfull[s], ph, abort, a.wait_ns))) break;
                    ctl->b_consumed = it + 1;
                    if (!(ok = mbar_wait(&ctl->afull[s], ph, abort, a.wait_ns))) break;
                    // the stage's A rows were written by the producers' cp.async (generic
                    // proxy); order them before the tensor cores' reads (async proxy)
                    fence_proxy_async_smem();
                    tc_fence_after();
                    // the stage's base descriptors once, then compile-time offsets
                    const uint64_t da = desc_k_sw128(smem_u32(smem + (size_t)s * G::STAGE));
                    const uint64_t db = da + (uint64_t)((3 * kPartBytes) >> 4);
#pragma unroll
                    for (int p = 0; p < 3; ++p)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mma_bf16(d, da + (uint64_t)((p * kPartBytes + k * 32) >> 4), db + (uint64_t)((k * 32) >> 4),
                                     idesc, (kc | p | k) ? 1u : 0u);
                    mma_commit(&ctl->empty[s]);
                }
                if (!ok) break;
                mma_commit(&ctl->tfull[acc]);  // also for a class without taps: nothing to wait for
                acc ^= 1u;
                if (acc == 0) acc_ph ^= 1u;
            }
            mma_commit(&ctl->drained);
            volatile int never = 0;
            mbar_wait(&ctl->drained, 0, &never, 200000000ull);
        }
    } else {
        // ------------------------------------------------ epilogue
        constexpr int CW = G::CW;
        const int q = warp & 3;  // TMEM lane quarter this warp may read
        const float ws = a.w_s ? *a.w_s : a.w_s_val;
        const float gsc = a.gmax_out ? *a.gmax_scale : 0.0f;
        const int HW = P.H * P.W;
        float gm = 0.0f;
        uint32_t acc = 0, acc_ph = 0;
        for (int t = blockIdx.x; t < P.tiles; t += gridDim.x) {
            const Class &C = P.cls[tile_class(P, t)];
            const int local = t - C.tile0, mt = local / P.ntn, n0 = (local - mt * P.ntn) * BN;
            const bool ok = mbar_wait_sleep(&ctl->tfull[acc], acc_ph, abort, a.wait_ns, 256);
            __syncwarp();  // reconverge before the warp-collective tcgen05.ld
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int m = mt * kRows + q * 32 + lane;
            const bool rv = m < a.B * C.Hc * C.Wc;
            int b = 0, y = 0, x = 0;
            if (rv) class_pixel(P, C, m, b, y, x);
            const i64 base = ((i64)b * P.Cin + n0) * HW + (i64)y * P.W + x;
            const bool any = C.kchunks > 0;
#pragma unroll 1
            for (int c0 = 0; c0 < BN && n0 + c0 < P.Cin; c0 += CW) {
                uint32_t v[CW];
                if (any) {
                    tmem_ld_cols<CW>(tbase + ((uint32_t)(q * 32) << 16) + acc * BN + c0, v);
                    tmem_ld_wait();
                }
                epilogue_cols<CW>(v, any, ws, a, base + (i64)c0 * HW, HW, P.Cin - n0 - c0, rv, gsc, gm);
            }
            tc_fence_before();
            __syncwarp();  // every lane's TMEM reads are done: one arrival per warp
            if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
            acc ^= 1u;
            if (acc == 0) acc_ph ^= 1u;
        }
        if (a.gmax_out) {
#pragma unroll
            for (int o = 16; o; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
            // non-negative floats order like their bit patterns
            if (lane == 0 && gm > 0.0f) atomicMax(reinterpret_cast<int *>(a.gmax_out), __float_as_int(gm));
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort) {
        // weight copies issued but never waited for must land before exit
        for (uint32_t i = ctl->b_consumed; i < ctl->b_issued; ++i) {
            volatile int never = 0;
            mbar_wait(&ctl->bfull[i % stages], (i / stages) & 1u, &never, 200000000ull);
        }
        atomicExch(&g_dgtc_error, 1);
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, G::TMEM_COLS);
    }
}


// ------------------------------------------------------------ halo tiling
// Stride-1 convs (plan.halo).  7 warps:
//   warp 0      halo producer: per (tile, chunk of KC output channels), one
//               bulk copy per (plane, 8-channel slab) of the tile's R
//               consecutive plane rows into an A stage laid out
//               [plane][slab][R rows][16 bytes] (no swizzle: a window of 128
//               rows starting at any row is a valid K-major operand with
//               SBO = 128 and LBO = R * 16).
//   warp 1      weight producer (lane 0): one bulk copy per (chunk, tap) of
//               the pre-laid-out weight block [KC / 8][BN][8].
//   warp 2      MMA issuer (lane 0): per (chunk, tap), 3 terms x KC / 16
//               K steps x mb row blocks of M = 128, N = BN, K = 16, the A
//               window shifted by the tap's offset; double-buffered TMEM
//               accumulators of mb x BN columns.
//   warps 3..10 epilogue, as the class kernel's, over the tile's positions
//               (gap positions are skipped): two warps per TMEM lane
//               quarter, each draining half of the tile's columns (BN >= 32).
constexpr int kHWarps = 11;
constexpr int kHThreads = 32 * kHWarps;
constexpr int kHEpi0 = 3;
constexpr int kMaxBStages = 16;

struct HCtl {
    uint64_t afull[2], aempty[2];
    uint64_t bfull[kMaxBStages], bempty[kMaxBStages];
    uint64_t tfull[2], tempty[2];
    uint64_t drained;
    uint32_t tmem_base;
    int abort;
    uint32_t a_issued, a_consumed, b_issued, b_consumed;
};

__host__ __device__ inline uint32_t halo_a_stage(const Halo &h) { return (3u * (h.KC >> 3) * h.R * 16 + 127) & ~127u; }
__host__ __device__ inline uint32_t halo_b_stage(const Plan &p) { return (uint32_t)p.BN * p.h.KC * 2; }
__host__ __device__ inline uint32_t halo_tmem_cols(const Plan &p) {
    uint32_t c = 32;
    while (c < (uint32_t)(p.h.nacc * p.h.mb * p.BN)) c <<= 1;
    return c;
}

// The MMA issuer of the halo kernel (one thread), for a compile-time channel
// chunk KC and tile height MB: per tile, per channel chunk (one halo stage),
// per tap of the tile's class (one weight stage), 3 split terms x KC / 16 K
// steps x MB row blocks of M = 128, N = BN, K = 16.  Every descriptor is a
// stage base plus offsets fixed before the loop (the per-term slab offsets
// are multiples of the run-time halo height R), so an MMA costs one add
// per operand.
template <int BN, int KC, int MB>
__device__ __forceinline__ void halo_mma_loop(const Plan &P, const Args &a, HCtl *ctl, uint32_t as0, uint32_t bs0,
                                              uint32_t tbase, uint32_t slab, uint32_t a_stage, uint32_t b_stage,
                                              volatile int *abort) {
    const Halo &h = P.h;
    constexpr uint32_t idesc = idesc_bf16(128, BN);
    constexpr int NSL = KC / 8, NK = KC / 16;
    const uint32_t a_lo0 = ((as0 >> 4) & 0x3FFFu) | desc_interleave_lo(slab);
    const uint32_t b_lo0 = ((bs0 >> 4) & 0x3FFFu) | desc_interleave_lo(BN * 16);
    const uint32_t hi = desc_interleave_hi(128);
    const uint32_t a_step = a_stage >> 4, b_step = b_stage >> 4, R = (uint32_t)h.R;
    uint32_t roff[3][NK];  // slab offset of (term, K step), in 16-byte units
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int kk = 0; kk < NK; ++kk) roff[p][kk] = (uint32_t)(p * NSL + 2 * kk) * R;
    uint32_t ia = 0, ib = 0, acc = 0, acc_ph = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < P.tiles && ok; t += gridDim.x) {
        if (!(ok = mbar_wait(&ctl->tempty[acc], acc_ph ^ 1u, abort, a.wait_ns))) break;
        tc_fence_after();
        const int k = tile_class(P, t);
        const int ntaps = P.cls[k].ntaps;
        const uint32_t d = tbase + acc * MB * BN;
        for (int c = 0; c < h.nchunks && ntaps > 0 && ok; ++c, ++ia) {
            const int sa = ia % h.sa;
            if (!(ok = mbar_wait(&ctl->afull[sa], (ia / h.sa) & 1u, abort, a.wait_ns))) break;
            ctl->a_consumed = ia + 1;
            tc_fence_after();
            const uint32_t a_lo = a_lo0 + sa * a_step;
            for (int tap = 0; tap < ntaps; ++tap, ++ib) {
                const int sb = ib % h.sb;
                if (!(ok = mbar_wait(&ctl->bfull[sb], (ib / h.sb) & 1u, abort, a.wait_ns))) break;
                ctl->b_consumed = ib + 1;
                tc_fence_after();
                const uint32_t al = a_lo + (uint32_t)h.off[k][tap], bl = b_lo0 + sb * b_step;
                const bool first = (c | tap) == 0;
#pragma unroll
                for (int p = 0; p < 3; ++p)
#pragma unroll
                    for (int kk = 0; kk < NK; ++kk) {
                        const uint64_t bd = desc_join(bl + kk * 2 * BN, hi);  // two slabs of BN rows x 16 bytes
#pragma unroll
                        for (int i = 0; i < MB; ++i)
                            mma_bf16(d + i * BN, desc_join(al + roff[p][kk] + i * 128, hi), bd, idesc,
                                     (first && p == 0 && kk == 0) ? 0u : 1u);
                    }
                mma_commit(&ctl->bempty[sb]);
            }
            if (!ok) break;
            mma_commit(&ctl->aempty[sa]);
        }
        if (!ok) break;
        mma_commit(&ctl->tfull[acc]);
        if (++acc == (uint32_t)h.nacc) acc = 0, acc_ph ^= 1u;
    }
    mma_commit(&ctl->drained);
    volatile int never = 0;
    mbar_wait(&ctl->drained, 0, &never, 200000000ull);
}

template <int BN>
__global__ void __launch_bounds__(kHThreads, 1) dgrad_halo_kernel(const __grid_constant__ Plan P, const Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Halo &h = P.h;
    const int nsl = h.KC >> 3, MT = 128 * h.mb;
    const uint32_t slab = (uint32_t)h.R * 16, a_stage = halo_a_stage(h), b_stage = halo_b_stage(P);
    uint8_t *As = smem;
    uint8_t *Bs = smem + (size_t)h.sa * a_stage;
    HCtl *ctl = reinterpret_cast<HCtl *>(Bs + (size_t)h.sb * b_stage);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tcols = halo_tmem_cols(P);

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ctl->afull[s], 1);
            mbar_init(&ctl->aempty[s], 1);
            mbar_init(&ctl->tfull[s], 1);
            mbar_init(&ctl->tempty[s], kHWarps - kHEpi0);  // one arrival per epilogue warp
        }
        for (int s = 0; s < h.sb; ++s) {
            mbar_init(&ctl->bfull[s], 1);
            mbar_init(&ctl->bempty[s], 1);
        }
        mbar_init(&ctl->drained, 1);
        ctl->abort = 0;
        ctl->a_issued = ctl->a_consumed = ctl->b_issued = ctl->b_consumed = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(&ctl->tmem_base, tcols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ctl->tmem_base;
    volatile int *abort = &ctl->abort;

    if (warp == 0) {
        // ------------------------------------------------ halo producer
        uint32_t ia = 0;
        bool run = true;
        for (int t = blockIdx.x; t < P.tiles && run; t += gridDim.x) {
            const Class &C = P.cls[tile_class(P, t)];
            if (C.ntaps == 0) continue;  // a phase without taps: the epilogue alone writes it
            const i64 row0 = (i64)((t - C.tile0) / P.ntn) * MT;  // plane row of the halo's first row
            for (int c = 0; c < h.nchunks; ++c, ++ia) {
                const int s = ia % h.sa;
                const uint32_t ph = (ia / h.sa) & 1u;
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&ctl->aempty[s], ph ^ 1u, abort, a.wait_ns);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    run = false;
                    break;
                }
                if (lane == 0) mbar_expect_tx(&ctl->afull[s], 3u * nsl * slab);
                __syncwarp();
                uint8_t *st = As + (size_t)s * a_stage;
                for (int idx = lane; idx < 3 * nsl; idx += 32) {
                    const int p = idx / nsl, sl = idx - p * nsl;
                    bulk_load(st + (size_t)idx * slab,
                              a.planes + p * a.plane_elems + ((i64)(c * nsl + sl) * h.rows + row0) * 8, slab,
                              &ctl->afull[s]);
                }
                __syncwarp();
                if (lane == 0) ctl->a_issued = ia + 1;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ weight producer
        if (lane == 0) {
            uint32_t ib = 0;
            bool run = true;
            for (int t = blockIdx.x; t < P.tiles && run; t += gridDim.x) {
                const Class &C = P.cls[tile_class(P, t)];
                const int nt = (t - C.tile0) % P.ntn, ntaps = C.ntaps;
                for (int c = 0; c < h.nchunks && run; ++c)
                    for (int tap = 0; tap < ntaps; ++tap, ++ib) {
                        const int s = ib % h.sb;
                        const uint32_t ph = (ib / h.sb) & 1u;
                        if (!mbar_wait(&ctl->bempty[s], ph ^ 1u, abort, a.wait_ns)) {
                            run = false;
                            break;
                        }
                        if (a.skip_weights) continue;
                        mbar_expect_tx(&ctl->bfull[s], b_stage);
                        bulk_load(Bs + (size_t)s * b_stage,
                                  a.wimg + ((i64)C.b_off + (i64)(nt * h.nchunks + c) * ntaps + tap) * b_stage,
                                  b_stage, &ctl->bfull[s]);
                        ctl->b_issued = ib + 1;
                    }
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------ MMA issuer (lane 0)
        if (lane == 0) {
            const uint32_t as0 = smem_u32(As), bs0 = smem_u32(Bs);
            switch (h.KC * 8 + h.mb) {
#define TRBA_HALO_LOOP(KC_, MB_)                                                                         \
    case KC_ * 8 + MB_:                                                                                  \
        if constexpr (MB_ * BN <= 384)                                                                   \
            halo_mma_loop<BN, KC_, MB_>(P, a, ctl, as0, bs0, tbase, slab, a_stage, b_stage, abort); \
        break;
                TRBA_HALO_LOOP(16, 1) TRBA_HALO_LOOP(16, 2) TRBA_HALO_LOOP(16, 3) TRBA_HALO_LOOP(16, 4)
                TRBA_HALO_LOOP(32, 1) TRBA_HALO_LOOP(32, 2) TRBA_HALO_LOOP(32, 3) TRBA_HALO_LOOP(32, 4)
                TRBA_HALO_LOOP(64, 1) TRBA_HALO_LOOP(64, 2) TRBA_HALO_LOOP(64, 3) TRBA_HALO_LOOP(64, 4)
#undef TRBA_HALO_LOOP
                default: *abort = 1; break;  // a tile the planner never makes
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        constexpr int CW = 16;  // accumulator columns per tcgen05.ld (BN >= 16)
        const int q = warp & 3;  // TMEM lane quarter this warp may read
        // columns of this warp: half of the tile's for BN >= 32, all of them
        // (first half) or none (second half) for BN = 16
        const int half = (warp - kHEpi0) >> 2;
        constexpr int HC = BN >= 32 ? BN / 2 : BN;
        const int cb = half * HC, ce = BN >= 32 ? cb + HC : (half ? 0 : BN);
        const float ws = a.w_s ? *a.w_s : a.w_s_val;
        const float gsc = a.gmax_out ? *a.gmax_scale : 0.0f;
        const int HW = P.H * P.W, HqWq = h.Hq * h.Wq;
        float gm = 0.0f;
        uint32_t acc = 0, acc_ph = 0;
        for (int t = blockIdx.x; t < P.tiles; t += gridDim.x) {
            const Class &C = P.cls[tile_class(P, t)];
            const int local = t - C.tile0, mt = local / P.ntn, n0 = (local - mt * P.ntn) * BN;
            const bool any = C.ntaps > 0;
            const bool ok = mbar_wait_sleep(&ctl->tfull[acc], acc_ph, abort, a.wait_ns, 256);
            __syncwarp();  // reconverge before the warp-collective tcgen05.ld
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            for (int i = 0; i < h.mb; ++i) {
                // position (b, i, j) of the class grid -> pixel (py + sH i, px + sW j)
                const i64 pos = (i64)mt * MT + i * 128 + q * 32 + lane;
                const int b = (int)(pos / HqWq), rem = (int)(pos - (i64)b * HqWq);
                const int ci = rem / h.Wq, cj = rem - ci * h.Wq;
                const bool rv = pos < h.mpos && ci < C.Hc && cj < C.Wc;
                const int y = C.py + (ci << P.lgSH), x = C.px + (cj << P.lgSW);
                const i64 base = ((i64)b * P.Cin + n0) * HW + (i64)y * P.W + x;
#pragma unroll 1
                for (int c0 = cb; c0 < ce && n0 + c0 < P.Cin; c0 += CW) {
                    uint32_t v[CW];
                    if (any) {
                        tmem_ld_cols<CW>(tbase + ((uint32_t)(q * 32) << 16) + (acc * h.mb + i) * BN + c0, v);
                        tmem_ld_wait();
                    }
                    epilogue_cols<CW>(v, any, ws, a, base + (i64)c0 * HW, HW, P.Cin - n0 - c0, rv, gsc, gm);
                }
            }
            tc_fence_before();
            __syncwarp();  // every lane's TMEM reads are done: one arrival per warp
            if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
            if (++acc == (uint32_t)h.nacc) acc = 0, acc_ph ^= 1u;
        }
        if (a.gmax_out) {
#pragma unroll
            for (int o = 16; o; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
            if (lane == 0 && gm > 0.0f) atomicMax(reinterpret_cast<int *>(a.gmax_out), __float_as_int(gm));
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort) {
        // copies issued but never waited for must land before exit
        volatile int never = 0;
        for (uint32_t i = ctl->a_consumed; i < ctl->a_issued; ++i)
            mbar_wait(&ctl->afull[i % h.sa], (i / h.sa) & 1u, &never, 200000000ull);
        for (uint32_t i = ctl->b_consumed; i < ctl->b_issued; ++i)
            mbar_wait(&ctl->bfull[i % h.sb], (i / h.sb) & 1u, &never, 200000000ull);
        atomicExch(&g_dgtc_error, 1);
    }
    __syncthreads();
    if (warp == 2) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, tcols);
    }
}
}  // namespace

// dy (NCHW f32) -> hi / mid / lo bf16 planes (NHWC), optionally scaled per
// output channel first.  Block: 32 pixels of one image; 32 channels at a time
// pass through a shared-memory transpose (reads coalesced along pixels,
// writes along channels).  C is a power of two >= 8.
__global__ void __launch_bounds__(256) split_nhwc_kernel(const float *__restrict__ dy,
                                                         const float *__restrict__ ws_co, int C, int HW,
                                                         uint16_t *__restrict__ planes, long long plane_elems) {
    __shared__ float tile[32][33];
    const int b = blockIdx.y, p0 = blockIdx.x * 32;
    const float *src = dy + (i64)b * C * HW;
    uint16_t *hi = planes + (i64)b * HW * C, *mid = hi + plane_elems, *lo = mid + plane_elems;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pl = threadIdx.x >> 3, cq = (threadIdx.x & 7) * 4;
    for (int c0 = 0; c0 < C; c0 += 32) {
        for (int cc = w; cc < 32; cc += 8) {
            const int c = c0 + cc, p = p0 + lane;
            float v = (c < C && p < HW) ? __ldg(src + (i64)c * HW + p) : 0.0f;
            if (ws_co && c < C) v = __fmul_rn(v, __ldg(ws_co + c));
            tile[cc][lane] = v;
        }
        __syncthreads();
        const int p = p0 + pl;
        if (p < HW && c0 + cq < C) {
            uint32_t h0, m0, l0, h1, m1, l1;
            split_pair(tile[cq][pl], tile[cq + 1][pl], h0, m0, l0);
            split_pair(tile[cq + 2][pl], tile[cq + 3][pl], h1, m1, l1);
            const i64 o = (i64)p * C + c0 + cq;
            *reinterpret_cast<uint2 *>(hi + o) = make_uint2(h0, h1);
            *reinterpret_cast<uint2 *>(mid + o) = make_uint2(m0, m1);
            *reinterpret_cast<uint2 *>(lo + o) = make_uint2(l0, l1);
        }
        __syncthreads();
    }
}

// dy (NCHW f32) -> hi / mid / lo bf16 planes in the halo layout
// [C / 8][rows][8]: plane row r holds position r + dmin of the padded grid
// (Hq x Wq per image), dy where the position is a real output pixel, zero in
// the gaps and guards (every row is written: the scratch is shared by convs
// of different geometry).  Thread: one row x one 8-channel slab; a warp reads
// 32 consecutive positions per channel and writes 512 contiguous bytes per
// plane.
__global__ void __launch_bounds__(256) split_halo_kernel(const float *__restrict__ dy,
                                                         const float *__restrict__ ws_co, int C, int Ho, int Wo,
                                                         int Hq, int Wq, int mpos, int dmin, int rows,
                                                         uint16_t *__restrict__ planes, long long plane_elems) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x, sl = blockIdx.y;
    if (r >= rows) return;
    const int pos = r + dmin;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.0f;
    if (pos >= 0 && pos < mpos) {
        const int HqWq = Hq * Wq, b = pos / HqWq, rem = pos - b * HqWq, yy = rem / Wq, xx = rem - yy * Wq;
        if (yy < Ho && xx < Wo) {
            const i64 HW = (i64)Ho * Wo;
            const float *src = dy + ((i64)b * C + sl * 8) * HW + (i64)yy * Wo + xx;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                v[e] = __ldg(src + e * HW);
                if (ws_co) v[e] = __fmul_rn(v[e], __ldg(ws_co + sl * 8 + e));
            }
        }
    }
    uint32_t hi[4], mid[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) split_pair(v[2 * e], v[2 * e + 1], hi[e], mid[e], lo[e]);
    uint16_t *o = planes + ((i64)sl * rows + r) * 8;
    *reinterpret_cast<uint4 *>(o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(o + plane_elems) = make_uint4(mid[0], mid[1], mid[2], mid[3]);
    *reinterpret_cast<uint4 *>(o + 2 * plane_elems) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Weight image from an int8 weight matrix [cout rows, w_ld] with K order
// (ci, kh, kw) (the ABI entry point's operand).
__global__ void image_from_wq_kernel(const __grid_constant__ Plan P, const int8_t *__restrict__ wq, int w_ld,
                                     uint8_t *__restrict__ wimg) {
    const i64 n = image_elements(P);
    GRID_LOOP(e, n) {
        int co;
        i64 dst;
        const int src = image_element(P, e, co, dst);
        const float v = src >= 0 ? (float)wq[(i64)co * w_ld + src] : 0.0f;
        *reinterpret_cast<__nv_bfloat16 *>(wimg + dst) = __float2bfloat16_rn(v);
    }
}

namespace {

// Raises a kernel's dynamic shared-memory limit to `smem` on the current
// device when the last value set there was lower.
template <typename K>
void ensure_smem(K kernel, size_t smem, int (&set)[64]) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || set[dev] >= (int)smem) return;
    TRBA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    set[dev] = (int)smem;
}

template <int BN>
void launch_bn(const Plan &p, const Args &a, int grid, cudaStream_t st) {
    using G = Geo<BN>;
    const size_t smem = 1024 + (size_t)a.stages * G::STAGE + sizeof(Ctl);
    static int set[64] = {};
    ensure_smem(dgrad_tc_kernel<BN>, smem, set);
    dgrad_tc_kernel<BN><<<grid, kThreads, smem, st>>>(p, a);
    TRBA_LAUNCH_CHECK();
}

size_t halo_smem(const Plan &p) {
    return 1024 + (size_t)p.h.sa * halo_a_stage(p.h) + (size_t)p.h.sb * halo_b_stage(p) + sizeof(HCtl);
}

template <int BN>
void launch_halo(const Plan &p, const Args &a, int grid, cudaStream_t st) {
    const size_t smem = halo_smem(p);
    static int set[64] = {};
    ensure_smem(dgrad_halo_kernel<BN>, smem, set);
    dgrad_halo_kernel<BN><<<grid, kHThreads, smem, st>>>(p, a);
    TRBA_LAUNCH_CHECK();
}

int stages_for(int BN) {
    const size_t stage = 3 * kPartBytes + (size_t)BN * kRowBytes;
    return (int)std::min<size_t>(kMaxStages, kSmemBudget / stage);
}

}  // namespace

namespace {

std::atomic<int> g_tiling_mb{0}, g_tiling_kc{0};

int halo_sms() {
    const int n = sm_count();
    return n > 0 ? n : 148;
}

// Shared-memory and TMEM fit of a halo tile of 128 * mb positions with KC
// channels per halo stage: halo rows R, stages (two halo stages when they
// fit with at least three weight stages, else one), accumulators (two when
// 2 x mb x BN columns fit TMEM).
struct HaloFit {
    bool ok;
    int R, sa, sb, nacc;
};

HaloFit halo_fit(const Plan &p, int mb, int KC) {
    HaloFit c{};
    const Halo &h = p.h;
    c.R = 128 * mb + h.dmax - h.dmin;
    Halo t = h;
    t.KC = KC, t.R = c.R;
    const size_t a = halo_a_stage(t), b = (size_t)p.BN * KC * 2;
    const size_t budget = kSmemBudget - sizeof(HCtl);
    c.nacc = 2 * mb * p.BN <= 512 ? 2 : 1;
    if (mb * p.BN > 384 || (size_t)c.R * 16 >= (1u << 18)) return c;
    if (2 * a + 3 * b <= budget) c.sa = 2;
    else if (a + 3 * b <= budget) c.sa = 1;
    else return c;
    c.sb = (int)std::min<size_t>(kMaxBStages, (budget - c.sa * a) / b);
    c.ok = true;
    return c;
}

// Preferred tile height: the smallest mb whose halo adds at most half a tile
// of rows (dmax - dmin <= 64 mb), else 4 (wide planes: the stem).  Measured
// on the model's convs at batch 512, taller tiles only pay where the halo
// is large: they halve the tile count (wave quantisation) without saving
// weight traffic that limits the kernel.
int halo_mb_pref(const Plan &p) {
    const int extra = p.h.dmax - p.h.dmin;
    for (int mb = 1; mb < 4; ++mb)
        if (extra <= 64 * mb) return mb;
    return 4;
}

// Halo geometry of a plan and its channel chunk KC (fixed here: the weight
// image depends on it; the tile height is set per batch): the largest KC
// (fewer, larger stages) whose stages fit two halo buffers at the preferred
// height, else the largest that fits at all, trying lower heights last.
// The padded slot (Hq, Wq) holds every row and column a class reads: reads
// above / left of the grid land in the previous slot's gap, reads below /
// right in this one's.  Leaves p.halo = 0 when the conv does not fit the
// tiling (Cout not a multiple of 16, padding >= kernel size, no fitting KC).
void make_halo(Plan &p) {
    if (p.Cout % 16 || p.pH < 0 || p.pW < 0 || p.pH >= p.kH || p.pW >= p.kW) return;
    Halo &h = p.h;
    int dh_lo = 0, dw_lo = 0, hq = p.Ho, wq = p.Wo;
    for (int k = 0; k < p.ncls; ++k) {
        const Class &C = p.cls[k];
        hq = std::max(hq, C.Hc);
        wq = std::max(wq, C.Wc);
        for (int t = 0; t < C.ntaps; ++t) {
            const int dh = (C.py + p.pH - C.kh[t]) / p.sH, dw = (C.px + p.pW - C.kw[t]) / p.sW;  // exact
            dh_lo = std::min(dh_lo, dh), dw_lo = std::min(dw_lo, dw);
            hq = std::max(hq, C.Hc + dh), wq = std::max(wq, C.Wc + dw);
        }
    }
    h.Hq = std::max(hq, p.Ho - dh_lo);
    h.Wq = std::max(wq, p.Wo - dw_lo);
    h.dmin = h.dmax = 0;
    h.taps = 0;
    for (int k = 0; k < p.ncls; ++k) {
        const Class &C = p.cls[k];
        for (int t = 0; t < C.ntaps; ++t) {
            const int o = (C.py + p.pH - C.kh[t]) / p.sH * h.Wq + (C.px + p.pW - C.kw[t]) / p.sW;
            h.dmin = std::min(h.dmin, o), h.dmax = std::max(h.dmax, o);
        }
        h.taps += C.ntaps;
    }
    for (int k = 0; k < p.ncls; ++k) {
        const Class &C = p.cls[k];
        for (int t = 0; t < C.ntaps; ++t)
            h.off[k][t] = (C.py + p.pH - C.kh[t]) / p.sH * h.Wq + (C.px + p.pW - C.kw[t]) / p.sW - h.dmin;
    }
    const int forced_mb = g_tiling_mb.load(), forced_kc = g_tiling_kc.load();
    const int mb0 = forced_mb > 0 ? forced_mb : halo_mb_pref(p);
    int kc = 0;
    for (int pass = 0; pass < 2 && !kc; ++pass)  // pass 0: two halo stages; pass 1: any fit
        for (int mb = mb0; mb >= (forced_mb > 0 ? mb0 : 1) && !kc; --mb)
            for (int KC = 64; KC >= 16 && !kc; KC /= 2) {
                if (p.Cout % KC || (forced_kc && KC != forced_kc)) continue;
                const HaloFit f = halo_fit(p, mb, KC);
                if (f.ok && (pass == 1 || f.sa == 2)) kc = KC;
            }
    if (!kc) return;
    h.KC = kc;
    h.nchunks = p.Cout / kc;
    int blocks = 0;  // weight blocks: (class, N tile, chunk, tap)
    for (int k = 0; k < p.ncls; ++k) {
        p.cls[k].b_off = blocks;
        blocks += p.ntn * h.nchunks * p.cls[k].ntaps;
    }
    p.halo = 1;
}

}  // namespace

bool make_plan(int Cin, int Cout, int H, int W, int kH, int kW, int sH, int sW, int pH, int pW, int Ho, int Wo,
               Plan &p) {
    auto lg2 = [](int v) {
        int l = 0;
        while ((1 << l) < v) ++l;
        return (1 << l) == v ? l : -1;
    };
    if (Cin <= 0 || Cout < 8 || lg2(Cout) < 0 || sH <= 0 || sW <= 0 || lg2(sH) < 0 || lg2(sW) < 0 ||
        sH * sW > kMaxClasses || H <= 0 || W <= 0 || Ho <= 0 || Wo <= 0)
        return false;
    p = Plan{};
    p.lgCout = lg2(Cout), p.lgSH = lg2(sH), p.lgSW = lg2(sW);
    p.Cin = Cin, p.Cout = Cout, p.H = H, p.W = W, p.Ho = Ho, p.Wo = Wo, p.kH = kH, p.kW = kW;
    p.sH = sH, p.sW = sW, p.pH = pH, p.pW = pW;
    if (Cin <= 16) p.BN = 16;
    else if (Cin <= 32) p.BN = 32;
    else if (Cin <= 64) p.BN = 64;
    else p.BN = 128;
    p.Npad = (Cin + p.BN - 1) / p.BN * p.BN;
    p.ntn = p.Npad / p.BN;
    int chunks = 0;
    for (int py = 0; py < sH; ++py)
        for (int px = 0; px < sW; ++px) {
            const int Hc = H > py ? (H - py + sH - 1) / sH : 0, Wc = W > px ? (W - px + sW - 1) / sW : 0;
            if (Hc == 0 || Wc == 0) continue;
            Class C{};
            C.py = py, C.px = px, C.Hc = Hc, C.Wc = Wc;
            for (int kh = 0; kh < kH; ++kh)
                for (int kw = 0; kw < kW; ++kw) {
                    if (((py + pH - kh) % sH + sH) % sH || ((px + pW - kw) % sW + sW) % sW) continue;
                    if (C.ntaps == kMaxTaps) return false;
                    C.kh[C.ntaps] = (int8_t)kh;
                    C.kw[C.ntaps] = (int8_t)kw;
                    ++C.ntaps;
                }
            C.kchunks = (C.ntaps * Cout + kChunk - 1) / kChunk;
            C.b_off = chunks;
            chunks += C.kchunks;
            p.cls[p.ncls++] = C;
        }
    p.total_chunks = chunks;
    if (p.ncls == 0) return false;
    if (g_tiling_mb.load() >= 0) make_halo(p);
    return true;
}

void set_tiling_override(int mb, int kc) {
    g_tiling_mb.store((mb >= 1 && mb <= 4) || mb < 0 ? mb : 0);
    g_tiling_kc.store(kc == 16 || kc == 32 || kc == 64 ? kc : 0);
}

void set_batch(Plan &p, int B) {
    p.B = B;
    if (p.halo) {
        Halo &h = p.h;
        h.mpos = (i64)B * h.Hq * h.Wq;
        const int forced = g_tiling_mb.load();
        // the preferred height (or the forced one), lowered while the KC of the
        // plan does not fit it or while it would leave SMs without a tile
        int best = forced > 0 ? forced : halo_mb_pref(p);
        while (best > 1 &&
               (!halo_fit(p, best, h.KC).ok ||
                (forced <= 0 && (h.mpos + 128 * best - 1) / (128 * best) * p.ntn * p.ncls < halo_sms())))
            --best;
        const HaloFit c = halo_fit(p, best, h.KC);
        h.mb = best, h.R = c.R, h.sa = c.sa, h.sb = c.sb, h.nacc = c.nacc;
        const i64 mtiles = (h.mpos + 128 * best - 1) / (128 * best);
        for (int k = 0; k < p.ncls; ++k) {  // every class covers the whole padded grid
            p.cls[k].tile0 = (int)(k * mtiles * p.ntn);
            p.cls[k].mtiles = (int)mtiles;
        }
        p.tiles = (int)(p.ncls * mtiles * p.ntn);
        h.rows = (mtiles - 1) * 128 * best + h.R;
        return;
    }
    int t = 0;
    for (int c = 0; c < p.ncls; ++c) {
        Class &C = p.cls[c];
        C.tile0 = t;
        C.mtiles = (int)(((i64)B * C.Hc * C.Wc + kRows - 1) / kRows);
        t += C.mtiles * p.ntn;
    }
    p.tiles = t;
}

namespace {
void launch_args(const Plan &p, const Args &a, cudaStream_t st) {
    const int grid = std::min(p.tiles, sm_count());
    if (p.halo) {
        switch (p.BN) {
            case 16: launch_halo<16>(p, a, grid, st); break;
            case 32: launch_halo<32>(p, a, grid, st); break;
            case 64: launch_halo<64>(p, a, grid, st); break;
            default: launch_halo<128>(p, a, grid, st); break;
        }
        return;
    }
    switch (p.BN) {
        case 16: launch_bn<16>(p, a, grid, st); break;
        case 32: launch_bn<32>(p, a, grid, st); break;
        case 64: launch_bn<64>(p, a, grid, st); break;
        default: launch_bn<128>(p, a, grid, st); break;
    }
}
}  // namespace

void launch(const Plan &p, const uint8_t *wimg, uint16_t *planes, const float *dy, const float *w_s, float w_s_val,
            const float *ws_co, const int8_t *mask_q, const float *add, float *gi, const float *gmax_scale,
            float *gmax_out, cudaStream_t st) {
    if (p.tiles <= 0) return;
    const int HoWo = p.Ho * p.Wo;
    const long long plane_elems = plane_elements(p);
    if (p.halo) {
        const Halo &h = p.h;
        split_halo_kernel<<<dim3((unsigned)((h.rows + 255) / 256), (unsigned)(p.Cout / 8)), 256, 0, st>>>(
            dy, ws_co, p.Cout, p.Ho, p.Wo, h.Hq, h.Wq, (int)h.mpos, h.dmin, (int)h.rows, planes, plane_elems);
    } else {
        split_nhwc_kernel<<<dim3((unsigned)((HoWo + 31) / 32), (unsigned)p.B), 256, 0, st>>>(dy, ws_co, p.Cout,
                                                                                          HoWo, planes, plane_elems);
    }
    TRBA_LAUNCH_CHECK();
    Args a{};
    a.planes = planes, a.plane_elems = plane_elems, a.wimg = wimg, a.w_s = w_s, a.w_s_val = w_s_val;
    a.mask_q = mask_q, a.add = add, a.gi = gi;
    a.gmax_scale = gmax_out ? gmax_scale : nullptr;
    a.gmax_out = gmax_scale ? gmax_out : nullptr;
    a.B = p.B;
    a.stages = stages_for(p.BN);
    a.wait_ns = 2000000000ull;
    a.skip_weights = 0;
    launch_args(p, a, st);
}

int error_poll(bool clear) {
    int v = 0;
    TRBA_CHECK(cudaDeviceSynchronize());
    TRBA_CHECK(cudaMemcpyFromSymbol(&v, g_dgtc_error, sizeof(int)));
    if (clear && v) {
        const int z = 0;
        TRBA_CHECK(cudaMemcpyToSymbol(g_dgtc_error, &z, sizeof(int)));
    }
    return v;
}

}  // namespace dgtc
}  // namespace trba

// -------------------------------------------------------------- C ABI --
namespace {
// Grow-only per-device buffer for the weight image and the dy planes of the
// ABI entry point (the fused training step keeps both in the model's arena).
std::mutex g_img_mu;
uint8_t *g_img[64] = {};
size_t g_img_bytes[64] = {};
}  // namespace

extern "C" int trba_conv_grad_input_i8_tc(const float *grad_out, const int8_t *weight_q, int w_ld, float w_scale,
                                          float *grad_input, int b, int cin, int h, int w, int cout, int kh, int kw,
                                          int sh, int sw, int ph, int pw, int ho, int wo, void *stream) {
    using namespace trba;
    if (b <= 0 || cin <= 0 || h <= 0 || w <= 0) return 0;
    dgtc::Plan p;
    if (!dgtc::make_plan(cin, cout, h, w, kh, kw, sh, sw, ph, pw, ho, wo, p)) {
        report_error(__FILE__, __LINE__,
                     "trba_conv_grad_input_i8_tc: unsupported conv (Cout and strides powers of two, Cout >= 8, at "
                     "most 4 stride phases and 16 taps per phase)", -1);
        return -1;
    }
    dgtc::set_batch(p, b);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return e != cudaSuccess ? (int)e : -1;
    const size_t img_bytes = ((size_t)dgtc::weight_image_bytes(p) + 255) & ~size_t(255);
    const size_t need = img_bytes + 3 * sizeof(uint16_t) * (size_t)dgtc::plane_elements(p);
    uint8_t *buf = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_img_mu);
        if (g_img_bytes[dev] < need) {
            if (g_img[dev]) TRBA_CHECK(cudaFree(g_img[dev]));
            g_img[dev] = nullptr;
            g_img_bytes[dev] = 0;
            e = cudaMalloc(&g_img[dev], need);
            if (e != cudaSuccess) {
                report_error(__FILE__, __LINE__, "trba_conv_grad_input_i8_tc: scratch allocation", (int)e);
                return (int)e;
            }
            g_img_bytes[dev] = need;
        }
        buf = g_img[dev];
    }
    cudaStream_t st = as_stream(stream);
    const long long n = dgtc::image_elements(p);
    dgtc::image_from_wq_kernel<<<grid_for(n), 256, 0, st>>>(p, weight_q, w_ld, buf);
    TRBA_LAUNCH_CHECK();
    const int before = trba_last_error();
    dgtc::launch(p, buf, reinterpret_cast<uint16_t *>(buf + img_bytes), grad_out, nullptr, w_scale, nullptr, nullptr,
                 nullptr, grad_input, nullptr, nullptr, st);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    const int after = trba_last_error();  // a launch error already reported in the sticky error mode
    return after != before ? (after ? after : -1) : 0;
}

// Bounded-wait self-test: small input-gradient launches of both tilings
// (a stride-2 conv on the class tiling, a stride-1 conv on the halo tiling)
// whose weight copies are never issued, so the MMA warp's first wait for them
// (and then every other role's) gives up after limit_ns; each kernel frees
// its tensor memory, sets the error word and returns.  Returns 1 when both
// kernels reported the give-up (and clears the word); the context stays
// usable.
namespace {
int wait_selftest_one(int stride, unsigned long long limit_ns, cudaStream_t st) {
    using namespace trba;
    dgtc::Plan p;
    const int ho = stride == 1 ? 8 : 4, wo = stride == 1 ? 16 : 8;
    if (!dgtc::make_plan(16, 16, 8, 16, 3, 3, stride, stride, 1, 1, ho, wo, p)) return -1;
    dgtc::set_batch(p, 2);
    // gi (2 x 16 x 8 x 16 floats), a zero weight image and zero dy planes
    const size_t n = 2 * 16 * 8 * 16;
    const size_t img = ((size_t)dgtc::weight_image_bytes(p) + 255) & ~size_t(255);
    const size_t planes = 3 * sizeof(uint16_t) * (size_t)dgtc::plane_elements(p);
    uint8_t *buf = nullptr;
    cudaError_t e = cudaMalloc(&buf, n * sizeof(float) + img + planes);
    if (e != cudaSuccess) return (int)e;
    TRBA_CHECK(cudaMemsetAsync(buf, 0, n * sizeof(float) + img + planes, st));
    dgtc::Args a{};
    a.gi = reinterpret_cast<float *>(buf);
    a.wimg = buf + n * sizeof(float);
    a.planes = reinterpret_cast<const uint16_t *>(buf + n * sizeof(float) + img);
    a.plane_elems = dgtc::plane_elements(p);
    a.w_s_val = 1.0f;
    a.B = p.B;
    a.stages = dgtc::stages_for(p.BN);
    a.wait_ns = limit_ns;
    a.skip_weights = 1;
    dgtc::launch_args(p, a, st);
    TRBA_CHECK(cudaStreamSynchronize(st));
    const int v = dgtc::error_poll(true);
    TRBA_CHECK(cudaFree(buf));
    return v;
}
}  // namespace

extern "C" int trba_tc_wait_selftest(unsigned long long limit_ns, void *stream) {
    cudaStream_t st = trba::as_stream(stream);
    const int a = wait_selftest_one(2, limit_ns, st);
    const int b = wait_selftest_one(1, limit_ns, st);
    return a == 1 && b == 1 ? 1 : (a != 1 ? a : b);
}

extern "C" void trba_tc_dgrad_tiling(int mb, int kc) { trba::dgtc::set_tiling_override(mb, kc); }

// Host-side plan of the tensor-core input gradient for a conv at batch b,
// for tests and tuning (no GPU work).  Writes up to n_out fields into out:
//   [0] halo  [1] BN  [2] Npad  [3] ntn  [4] tiles  [5] taps of all classes
//   halo plans only:
//   [6] KC  [7] nchunks  [8] mb  [9] R  [10] sa  [11] sb  [12] Hq  [13] Wq
//   [14] dmin  [15] mpos  [16] rows  [17] plane elements  [18] image bytes
//   [19] shared-memory bytes  [20] TMEM columns  [21] classes, then per
//   class: py, px, Hc, Wc, ntaps, tile0, mtiles, first weight block, and
//   per tap kh, kw, offset from the halo's first row
// Returns the number of fields the plan has, or -1 when the conv is not served.
extern "C" int trba_tc_dgrad_plan(int b, int cin, int h, int w, int cout, int kh, int kw, int sh, int sw, int ph,
                                  int pw, int ho, int wo, long long *out, int n_out) {
    using namespace trba::dgtc;
    Plan p;
    if (b <= 0 || !make_plan(cin, cout, h, w, kh, kw, sh, sw, ph, pw, ho, wo, p)) return -1;
    set_batch(p, b);
    std::vector<long long> f = {p.halo, p.BN, p.Npad, p.ntn, p.tiles, p.halo ? p.h.taps : 0};
    if (p.halo) {
        const Halo &hh = p.h;
        for (long long x : {(long long)hh.KC, (long long)hh.nchunks, (long long)hh.mb, (long long)hh.R,
                            (long long)hh.sa, (long long)hh.sb, (long long)hh.Hq, (long long)hh.Wq,
                            (long long)hh.dmin, hh.mpos, hh.rows, plane_elements(p), weight_image_bytes(p),
                            (long long)halo_smem(p), (long long)halo_tmem_cols(p), (long long)p.ncls})
            f.push_back(x);
        for (int k = 0; k < p.ncls; ++k) {
            const Class &C = p.cls[k];
            for (long long x : {C.py, C.px, C.Hc, C.Wc, C.ntaps, C.tile0, C.mtiles, C.b_off}) f.push_back(x);
            for (int t = 0; t < C.ntaps; ++t) {
                f.push_back(C.kh[t]);
                f.push_back(C.kw[t]);
                f.push_back(hh.off[k][t]);
            }
        }
    }
    for (int i = 0; i < (int)f.size() && i < n_out; ++i) out[i] = f[i];
    return (int)f.size();
}
