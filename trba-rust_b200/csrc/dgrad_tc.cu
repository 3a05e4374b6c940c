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
    uint64_t tempty[2];          // accumulator drained (128 epilogue arrivals)
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
    static constexpr int CW = BN < 32 ? BN : 32;  // accumulator columns per tcgen05.ld
};

template <int CW>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[CW]) {
    if constexpr (CW == 16) tmem_ld_32x32b_x16(taddr, v);
    else tmem_ld_32x32b_x32(taddr, v);
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
            mbar_init(&ctl->tempty[i], kEpiWarps * 32);
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
                    const uint32_t st = smem_u32(smem + (size_t)s * G::STAGE);
                    const uint32_t b0 = st + 3 * kPartBytes;
#pragma unroll
                    for (int p = 0; p < 3; ++p)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mma_bf16(d, desc_k_sw128(st + p * kPartBytes + k * 32), desc_k_sw128(b0 + k * 32), idesc,
                                     (kc | p | k) ? 1u : 0u);
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
#pragma unroll
                for (int j = 0; j < CW; ++j) {
                    if (rv && n0 + c0 + j < P.Cin) {
                        const i64 i = base + (i64)(c0 + j) * HW;
                        float val = any ? fmul(__uint_as_float(v[j]), ws) : 0.0f;
                        if (a.mask_q) val = a.mask_q[i] > 0 ? val : 0.0f;
                        if (a.add) val = fadd(val, a.add[i]);
                        a.gi[i] = val;
                        gm = fmaxf(gm, fabsf(fmul(val, gsc)));
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&ctl->tempty[acc]);
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

// Weight image from an int8 weight matrix [cout rows, w_ld] with K order
// (ci, kh, kw) (the ABI entry point's operand).
__global__ void image_from_wq_kernel(const __grid_constant__ Plan P, const int8_t *__restrict__ wq, int w_ld,
                                     uint8_t *__restrict__ wimg) {
    const i64 n = (i64)P.total_chunks * P.Npad * kChunk;
    GRID_LOOP(e, n) {
        int gc, row, kl, co;
        image_entry(P, e, gc, row, kl);
        const int src = image_source(P, gc, row, kl, co);
        const float v = src >= 0 ? (float)wq[(i64)co * w_ld + src] : 0.0f;
        *reinterpret_cast<__nv_bfloat16 *>(wimg + image_offset(gc, row, kl, P.Npad)) = __float2bfloat16_rn(v);
    }
}

namespace {

template <int BN>
void launch_bn(const Plan &p, const Args &a, int grid, cudaStream_t st) {
    using G = Geo<BN>;
    const size_t smem = 1024 + (size_t)a.stages * G::STAGE + sizeof(Ctl);
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        TRBA_CHECK(cudaFuncSetAttribute(dgrad_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr[dev] = true;
    }
    dgrad_tc_kernel<BN><<<grid, kThreads, smem, st>>>(p, a);
    TRBA_LAUNCH_CHECK();
}

int stages_for(int BN) {
    const size_t stage = 3 * kPartBytes + (size_t)BN * kRowBytes;
    return (int)std::min<size_t>(kMaxStages, kSmemBudget / stage);
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
    return p.ncls > 0;
}

void set_batch(Plan &p, int B) {
    p.B = B;
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
    split_nhwc_kernel<<<dim3((unsigned)((HoWo + 31) / 32), (unsigned)p.B), 256, 0, st>>>(dy, ws_co, p.Cout, HoWo,
                                                                                      planes, plane_elems);
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
    const long long n = (long long)p.total_chunks * p.Npad * dgtc::kChunk;
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

// Bounded-wait self-test: one small input-gradient launch whose weight copies
// are never issued, so the MMA warp's first wait for them (and then every
// other role's) gives up after limit_ns; the kernel frees its tensor memory,
// sets the error word and returns.  Returns the error word (1 expected) and
// clears it; the context stays usable.
extern "C" int trba_tc_wait_selftest(unsigned long long limit_ns, void *stream) {
    using namespace trba;
    dgtc::Plan p;
    if (!dgtc::make_plan(16, 16, 8, 16, 3, 3, 1, 1, 1, 1, 8, 16, p)) return -1;
    dgtc::set_batch(p, 2);
    // gi (2 x 16 x 8 x 16 floats), a zero weight image and zero dy planes
    const size_t n = 2 * 16 * 8 * 16;
    const size_t img = ((size_t)dgtc::weight_image_bytes(p) + 255) & ~size_t(255);
    const size_t planes = 3 * sizeof(uint16_t) * (size_t)dgtc::plane_elements(p);
    uint8_t *buf = nullptr;
    cudaError_t e = cudaMalloc(&buf, n * sizeof(float) + img + planes);
    if (e != cudaSuccess) return (int)e;
    cudaStream_t st = as_stream(stream);
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
