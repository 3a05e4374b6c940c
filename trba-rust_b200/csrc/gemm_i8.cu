// int8 GEMM on B200 tensor cores: C[M,N] s32 = A[M,K] . Bt[N,K]^T with
// tcgen05 kind::i8 (reference contract of launch_gemm_int8:
// cuda/kernels.cu:227-250 of the checked-out tree — row-major operands,
// leading dimension align16(K), compact C).
//
// Design (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0 lane 0 : TMA producer. For each 128 x BN output tile (and K
//                   split) it streams 128-byte K slices of A (128 rows) and
//                   B (BN rows) into a STAGES-deep ring of 128B-swizzled
//                   shared-memory stages.
//   warp 1 lane 0 : MMA issuer. Four tcgen05.mma (M=128, N=BN, K=32) per
//                   stage into one of two TMEM accumulators, so the epilogue
//                   of tile i overlaps the MMAs of tile i+1.
//   warps 2..5    : epilogue. tcgen05.ld 32 columns at a time (each thread
//                   owns one output row) and hands them to an epilogue policy:
//                     EpiS32       s32 store (launch_gemm_int8)
//                     EpiS32Atomic s32 atomicAdd, for split-K (exact: integer
//                                  addition is associative)
//                     EpiConvF32   conv forward: x = acc * (s_in * w_s) written
//                                  NCHW, plus per-channel sum / sum of squares
//                                  of x in f64 for the BatchNorm statistics.
// Tensor maps cover exactly [M, K] and [N, K]: TMA zero-fills every
// out-of-range row and column, so the kernel never reads the operands'
// padding and needs no tail handling in the main loop.
//
// Every mbarrier wait is bounded (2 s): on a timeout the CTA raises an abort
// flag, every role leaves its loop, in-flight loads are drained, TMEM is
// freed and the device error word g_tc_error is set for the host to read.
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "dgrad_tc.cuh"
#include "gemm_i8.cuh"
#include "trba_backend.h"
#include "tc_primitives.cuh"

using namespace trba;
using namespace trba::tc;

__device__ int g_tc_error = 0;

namespace {

constexpr int BM = 128;   // UMMA M (cta_group::1)
constexpr int BK = 128;   // bytes of K per stage = one 128B swizzle row
constexpr int UK = 32;    // K of one kind::i8 MMA
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, splitting the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxN = 512;  // widest N an epilogue with per-column state supports

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // two accumulators (power of two >= 64)
    static constexpr int EPI_SMEM = 2 * kMaxN * 8;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 512 + EPI_SMEM;
    static_assert(kEpiWarps * 1024 <= EPI_SMEM, "EpiS32 stages 1 KB per epilogue warp");
};

struct Ctl {  // lives after the stage ring in shared memory
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t afull[8];  // implicit-GEMM conv: the gathered A rows of a stage have landed
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drained;
    uint32_t tmem_base;
    int abort;
    uint32_t issued;    // stage loads issued by the producer
    uint32_t consumed;  // stage loads whose data the MMA warp waited for
};

// Sum of a[] over the 32 lanes for each of 32 columns: afterwards lane l
// holds the total of column l (butterfly reduce-scatter, 31 shuffles).
__device__ __forceinline__ double reduce_scatter32(double (&a)[32], int lane) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool upper = lane & s;
#pragma unroll
        for (int j = 0; j < s; ++j) {
            const double send = upper ? a[j] : a[j + s];
            const double keep = upper ? a[j + s] : a[j];
            a[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
    return a[0];
}

// ------------------------------------------------------------ epilogues --
struct EpiS32 {
    int32_t *C;
    int ldc;
    bool vec4;  // C rows are 16-byte aligned and N % 4 == 0
    __device__ void init(double *) {}
    // Each lane holds 32 consecutive columns of its own row.  Written as they
    // are, one 16-byte store per lane touches 32 rows: every 32-byte sector
    // is written in two halves by two instructions.  Instead the warp's 32
    // rows pass 8 columns at a time through its own 1 KB of shared memory
    // (the epilogue's scratch, unused by this policy): two lanes then write
    // one row's 8 columns, so every store instruction writes 16 whole
    // sectors.  Pieces are XOR-swizzled by row so neither side conflicts.
    __device__ void store(int row, int col, int M, int N, const uint32_t (&v)[32], int lane, double *sm) {
        if (!(vec4 && col + 32 <= N)) {  // warp-uniform (col and N are)
            if (row >= M) return;
            int32_t *crow = C + (i64)row * ldc;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col + j < N) crow[col + j] = (int32_t)v[j];
            return;
        }
        uint8_t *buf = reinterpret_cast<uint8_t *>(sm) + (size_t)((threadIdx.x >> 5) - 2) * 1024;
        const int row0 = row - lane;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
                *reinterpret_cast<uint4 *>(buf + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4)) =
                    make_uint4(v[8 * p + 4 * h], v[8 * p + 4 * h + 1], v[8 * p + 4 * h + 2], v[8 * p + 4 * h + 3]);
            __syncwarp();
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int k = lane + 32 * t, r = k >> 1, half = k & 1;
                const uint4 w = *reinterpret_cast<const uint4 *>(buf + r * 32 + ((half ^ ((r >> 2) & 1)) << 4));
                if (row0 + r < M)
                    *reinterpret_cast<uint4 *>(C + (i64)(row0 + r) * ldc + col + 8 * p + 4 * half) = w;
            }
            __syncwarp();
        }
    }
    __device__ void finish(double *, int) {}
};

struct EpiS32Atomic {
    int32_t *C;
    int ldc;
    __device__ void init(double *) {}
    // Integer atomics, exact in any order.  As in EpiS32, the warp's 32 rows
    // pass 8 columns at a time through its 1 KB of shared memory, so that one
    // atomic instruction covers 8 consecutive columns of 4 rows (4 sectors)
    // instead of one column of 32 rows (32 lines).
    __device__ void store(int row, int col, int M, int N, const uint32_t (&v)[32], int lane, double *sm) {
        uint8_t *buf = reinterpret_cast<uint8_t *>(sm) + (size_t)((threadIdx.x >> 5) - 2) * 1024;
        const int row0 = row - lane, c = lane & 7;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
                *reinterpret_cast<uint4 *>(buf + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4)) =
                    make_uint4(v[8 * p + 4 * h], v[8 * p + 4 * h + 1], v[8 * p + 4 * h + 2], v[8 * p + 4 * h + 3]);
            __syncwarp();
            const int n = col + 8 * p + c;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 4 * i + (lane >> 3);  // r >> 2 == i
                const uint32_t val =
                    *reinterpret_cast<const uint32_t *>(buf + r * 32 + ((((c >> 2) ^ (i & 1))) << 4) + (c & 3) * 4);
                if (row0 + r < M && n < N && val != 0u) atomicAdd(C + (i64)(row0 + r) * ldc + n, (int32_t)val);
            }
            __syncwarp();
        }
    }
    __device__ void finish(double *, int) {}
};

struct EpiConvF32 {
    float *x;            // NCHW output, row r = b*HW + p, column = channel
    const float *s_in;   // device scalar: activation scale of the conv input
    const float *w_s;    // weight scale: device scalar, or [N] per output channel
    int per_channel;
    double *bn_acc;      // [2*N]: per-channel sum, then sum of squares (f64)
    int HW;
    __device__ __forceinline__ float scale_of(int n) const { return fmul(*s_in, per_channel ? w_s[n] : *w_s); }
    __device__ void init(double *sm) {
        for (int i = threadIdx.x - 64; i < 2 * kMaxN; i += blockDim.x - 64) sm[i] = 0.0;
    }
    __device__ void store(int row, int col, int M, int N, const uint32_t (&v)[32], int lane, double *sm) {
        const bool rv = row < M;
        const int b = rv ? row / HW : 0, p = rv ? row - b * HW : 0;
        // the scales are read before any store (a store to x could alias
        // them as far as the compiler knows, which would make every column
        // wait for the previous column's store)
        float sc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) sc[j] = scale_of(col + j < N ? col + j : N - 1);
        double s[32], q[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float val = fmul((float)(int32_t)v[j], sc[j]);
            const bool ok = rv && col + j < N;
            if (ok) x[((i64)b * N + col + j) * HW + p] = val;
            s[j] = ok ? (double)val : 0.0;
            q[j] = ok ? (double)val * (double)val : 0.0;
        }
        const double cs = reduce_scatter32(s, lane);
        const double cq = reduce_scatter32(q, lane);
        if (col + lane < N) {
            atomicAdd(sm + col + lane, cs);
            atomicAdd(sm + kMaxN + col + lane, cq);
        }
    }
    __device__ void finish(double *sm, int N) {
        for (int i = threadIdx.x - 64; i < N; i += blockDim.x - 64) {
            if (sm[i] != 0.0) atomicAdd(bn_acc + i, sm[i]);
            if (sm[kMaxN + i] != 0.0) atomicAdd(bn_acc + N + i, sm[kMaxN + i]);
        }
    }
    // Row accumulation (BN = 32, one n block): an epilogue warp drains the
    // same 16 columns of every tile it takes; each lane adds its rows'
    // values and squares to f64 partial sums held in registers, and the warp
    // reduces them across lanes once, at the end.
    static constexpr bool kRowAccum = true;
    struct Accum {
        double s[16], q[16];
    };
    __device__ void acc_init(Accum &a) {
#pragma unroll
        for (int j = 0; j < 16; ++j) a.s[j] = a.q[j] = 0.0;
    }
    // columns [col, col + 16) of the tile row, taken from v[16 hi + j]
    __device__ void store_acc(int row, int col, int M, int N, const uint32_t (&v)[32], bool hi, Accum &a) {
        if (row >= M) return;
        const int b = row / HW, p = row - b * HW;
        float *xp = x + ((i64)b * N + col) * HW + p;
        float sc[16];  // read before any store, as in store()
#pragma unroll
        for (int j = 0; j < 16; ++j) sc[j] = scale_of(col + j < N ? col + j : N - 1);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (col + j < N) {
                const float val = fmul((float)(int32_t)(hi ? v[16 + j] : v[j]), sc[j]);
                xp[(i64)j * HW] = val;
                const double d = (double)val;
                a.s[j] += d;
                a.q[j] = fma(d, d, a.q[j]);
            }
        }
    }
    __device__ void acc_flush(Accum &a, int col, int N, int lane, double *sm) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            a.s[j] += __shfl_xor_sync(0xffffffffu, a.s[j], 16);
            a.q[j] += __shfl_xor_sync(0xffffffffu, a.q[j], 16);
        }
        // reduce-scatter over the 16 lanes left: lane l ends with column l & 15
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1) {
            const bool upper = lane & w;
#pragma unroll
            for (int j = 0; j < w; ++j) {
                const double ss = upper ? a.s[j] : a.s[j + w], ks = upper ? a.s[j + w] : a.s[j];
                const double sq = upper ? a.q[j] : a.q[j + w], kq = upper ? a.q[j + w] : a.q[j];
                a.s[j] = ks + __shfl_xor_sync(0xffffffffu, ss, w);
                a.q[j] = kq + __shfl_xor_sync(0xffffffffu, sq, w);
            }
        }
        if (lane < 16 && col + lane < N) {
            atomicAdd(sm + col + lane, a.s[0]);
            atomicAdd(sm + kMaxN + col + lane, a.q[0]);
        }
    }
};

template <class Epi, class = void>
struct HasRowAccum {
    static constexpr bool value = false;
};
template <class Epi>
struct HasRowAccum<Epi, decltype(void(Epi::kRowAccum))> {
    static constexpr bool value = Epi::kRowAccum;
};

// Division by a per-call divisor b with r = RN(1/b) precomputed on the
// host: Markstein's FMA division (q = RN(a r), e = a - b q exact by FMA,
// RN(q + e r)), which gives RN(a / b) for normal a and b whenever q is a
// faithful quotient and r approximates 1/b within a relative 2^-24, with no
// underflow or overflow (Handbook of Floating-Point Arithmetic, Muller et
// al., the theorem on Markstein's division).  The host takes this path only
// for 2^-90 <= |b| <= 2^90, where every quotient of an s32 accumulator by b
// is a normal float; trba_requant_division_check compares it with the
// IEEE division for every s32 accumulator value.
__device__ __forceinline__ float div_by(float a, float b, float r) {
    const float q = __fmul_rn(a, r);
    const float e = __fmaf_rn(-q, b, a);
    return __fmaf_rn(e, r, q);
}

// Fused inference epilogue of the conv path (cuda/kernels.cu:434-466,
// launch_conv_epilogue): out[r, n] = rint(clamp(max(acc/div + bias[n], 0) *
// mul, +-127)) as int8, row-major [M, ldo].
struct EpiRequantI8 {
    int8_t *out;
    int ldo;
    const float *bias;
    float div, mul;
    bool vec;     // out rows 16-byte aligned and N % 16 == 0
    float rdiv;   // RN(1 / div) when fast_div
    bool fast_div;
    __device__ void init(double *) {}
    __device__ void store(int row, int col, int M, int N, const uint32_t (&v)[32], int lane, double *sm) {
        int8_t *orow = out + (i64)row * ldo;  // rows >= M compute but never store
        // the 32 columns' biases (the same for every lane: broadcast loads)
        float bv[32];
        if (col + 32 <= N && (reinterpret_cast<uintptr_t>(bias + col) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 b4 = reinterpret_cast<const float4 *>(bias + col)[j];
                bv[4 * j] = b4.x, bv[4 * j + 1] = b4.y, bv[4 * j + 2] = b4.z, bv[4 * j + 3] = b4.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) bv[j] = bias[col + j < N ? col + j : N - 1];
        }
        uint32_t packed[8];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float a = (float)(int32_t)v[j];
            float t = fadd(fast_div ? div_by(a, div, rdiv) : fdiv(a, div), bv[j]);
            t = fmul(fmaxf(t, 0.0f), mul);
            t = fminf(fmaxf(t, -127.0f), 127.0f);
            const uint32_t q = (uint32_t)(uint8_t)(int8_t)rint_even(t);
            if ((j & 3) == 0) packed[j >> 2] = 0u;
            packed[j >> 2] |= q << (8 * (j & 3));
        }
        if (vec && col + 32 <= N) {
            // the row's 32 bytes are one sector: the warp's 32 rows pass
            // through its 1 KB of shared memory so that two lanes write one
            // row and every store instruction writes 16 whole sectors
            uint8_t *buf = reinterpret_cast<uint8_t *>(sm) + (size_t)((threadIdx.x >> 5) - 2) * 1024;
            const int row0 = row - lane;
#pragma unroll
            for (int h = 0; h < 2; ++h)
                *reinterpret_cast<uint4 *>(buf + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4)) =
                    make_uint4(packed[4 * h], packed[4 * h + 1], packed[4 * h + 2], packed[4 * h + 3]);
            __syncwarp();
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int k = lane + 32 * t, r = k >> 1, half = k & 1;
                const uint4 w = *reinterpret_cast<const uint4 *>(buf + r * 32 + ((half ^ ((r >> 2) & 1)) << 4));
                if (row0 + r < M) *reinterpret_cast<uint4 *>(out + (i64)(row0 + r) * ldo + col + 16 * half) = w;
            }
            __syncwarp();
        } else {
            if (row >= M) return;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col + j < N) orow[col + j] = (int8_t)((packed[j >> 2] >> (8 * (j & 3))) & 0xffu);
        }
    }
    __device__ void finish(double *, int) {}
};

// Dequantising epilogue with per-output-channel weight scales:
// out[r, n] = act((float)acc * (a_scale * w_scale[n]) [+ bias[n]]), f32
// row-major [M, ldo]; act = ReLU when relu, identity otherwise.
struct EpiDequantF32 {
    float *out;
    int ldo;
    const float *w_scale;
    const float *bias;  // may be null
    float a_scale;
    int relu;
    bool vec;  // out rows 16-byte aligned and N % 4 == 0
    __device__ void init(double *) {}
    __device__ void store(int row, int col, int M, int N, const uint32_t (&v)[32], int lane, double *sm) {
        float r[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int n = col + j < N ? col + j : N - 1;
            float t = fmul((float)(int32_t)v[j], fmul(a_scale, w_scale[n]));
            if (bias) t = fadd(t, bias[n]);
            r[j] = relu ? fmaxf(t, 0.0f) : t;
        }
        if (vec && col + 32 <= N) {  // warp-uniform: whole sectors per store, as in EpiS32
            uint8_t *buf = reinterpret_cast<uint8_t *>(sm) + (size_t)((threadIdx.x >> 5) - 2) * 1024;
            const int row0 = row - lane;
#pragma unroll
            for (int p = 0; p < 4; ++p) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    *reinterpret_cast<float4 *>(buf + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4)) =
                        make_float4(r[8 * p + 4 * h], r[8 * p + 4 * h + 1], r[8 * p + 4 * h + 2], r[8 * p + 4 * h + 3]);
                __syncwarp();
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const int k = lane + 32 * t, rr = k >> 1, half = k & 1;
                    const float4 w = *reinterpret_cast<const float4 *>(buf + rr * 32 + ((half ^ ((rr >> 2) & 1)) << 4));
                    if (row0 + rr < M) *reinterpret_cast<float4 *>(out + (i64)(row0 + rr) * ldo + col + 8 * p + 4 * half) = w;
                }
                __syncwarp();
            }
        } else {
            if (row >= M) return;
            float *orow = out + (i64)row * ldo;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col + j < N) orow[col + j] = r[j];
        }
    }
    __device__ void finish(double *, int) {}
};

struct Shape {
    int M, N, K;
    int splits;        // K splits (1 = none)
    int kb_per_split;  // K blocks of 128 per split
};

// Where the A operand comes from.
//   TmaA       a row-major int8 matrix read through the A tensor map.
//   ConvGather the implicit-GEMM conv forward: A[r, k] for output pixel
//              r = (b, oy, ox) and k = (ky * kw + kx) * Cin + ci is read
//              straight from NHWC int8 activations by kGatherWarps extra
//              warps with 16-byte cp.async (zero-filled where the tap falls
//              on the conv's zero padding), written into the stage in the
//              layout TMA's 128-byte swizzle gives, so the im2col matrix is
//              never materialised.  Integer accumulation makes the K order
//              irrelevant: the s32 results equal im2col + GEMM exactly.
struct TmaA {
    static constexpr bool kGather = false;
};
struct ConvGather {
    static constexpr bool kGather = true;
    const int8_t *x;  // [B, H, W, Cin], 16-byte aligned; Cin = 1 << lgC >= 16
    int H, W, lgC, kh, kw, sh, sw, ph, pw, Wo, HoWo;
};
constexpr int kGatherWarps = 2;
template <class Src>
constexpr int threads_for() {
    return kThreads + (Src::kGather ? 32 * kGatherWarps : 0);
}

template <int BN, class Epi, class Src = TmaA>
__global__ void __launch_bounds__(threads_for<Src>(), 1)
gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Shape sh,
                  Epi epi, Src src = Src()) {
    using G = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + G::STAGES * G::A_BYTES;
    Ctl *ctl = reinterpret_cast<Ctl *>(smem + G::STAGES * G::STAGE_BYTES);
    double *epi_sm = reinterpret_cast<double *>(smem + G::STAGES * G::STAGE_BYTES + 512);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = sh.M, N = sh.N, K = sh.K;
    const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles * sh.splits, kblocks = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
            if constexpr (Src::kGather) mbar_init(&ctl->afull[s], 32 * kGatherWarps);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&ctl->tfull[a], 1);
            mbar_init(&ctl->tempty[a], kEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(&ctl->drained, 1);
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        fence_barrier_init();
        if constexpr (!Src::kGather) tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp >= 2) epi.init(epi_sm);
    if (warp == 1) {
        tmem_alloc(&ctl->tmem_base, G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ctl->tmem_base;
    volatile int *abort = &ctl->abort;

    // tile t -> (split, m block, n block); n fastest so CTAs working at the
    // same time share the A block through L2.
    auto tile_coords = [&](int t, int &m0, int &n0, int &kb0, int &kb1) {
        const int per_split = m_tiles * n_tiles;
        const int sp = t / per_split, r = t - sp * per_split;
        m0 = (r / n_tiles) * BM;
        n0 = (r % n_tiles) * BN;
        kb0 = sp * sh.kb_per_split;
        kb1 = min(kblocks, kb0 + sh.kb_per_split);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t it = 0;
            for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
                int m0, n0, kb0, kb1;
                tile_coords(t, m0, n0, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % G::STAGES;
                    const uint32_t ph = (it / G::STAGES) & 1u;
                    if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort)) break;
                    if constexpr (Src::kGather) {  // A comes from the gather warps
                        mbar_expect_tx(&ctl->full[s], G::B_BYTES);
                    } else {
                        mbar_expect_tx(&ctl->full[s], G::STAGE_BYTES);
                        tma_load_2d(sA + s * G::A_BYTES, &tmA, &ctl->full[s], kb * BK, m0);
                    }
                    tma_load_2d(sB + s * G::B_BYTES, &tmB, &ctl->full[s], kb * BK, n0);
                    ctl->issued = it + 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_i8(BM, BN);
            uint32_t it = 0, acc = 0, acc_ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                int m0, n0, kb0, kb1;
                tile_coords(t, m0, n0, kb0, kb1);
                if (!(ok = mbar_wait(&ctl->tempty[acc], acc_ph ^ 1u, abort))) break;
                tc_fence_after();
                const uint32_t d = tbase + acc * BN;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % G::STAGES;
                    const uint32_t ph = (it / G::STAGES) & 1u;
                    if (!(ok = mbar_wait(&ctl->full[s], ph, abort))) break;
                    ctl->consumed = it + 1;
                    if constexpr (Src::kGather) {
                        if (!(ok = mbar_wait(&ctl->afull[s], ph, abort))) break;
                        // the gathered rows were written by cp.async (generic proxy):
                        // order them before the tensor cores' reads (async proxy)
                        fence_proxy_async_smem();
                    }
                    tc_fence_after();
                    // the stage's base descriptors once, then compile-time K offsets
                    // (one add per MMA: a descriptor rebuilt per MMA halves the issue rate)
                    const uint64_t da = desc_k_sw128(smem_u32(sA + s * G::A_BYTES));
                    const uint64_t db = desc_k_sw128(smem_u32(sB + s * G::B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UK; ++k)
                        mma_i8(d, da + (uint64_t)((k * UK) >> 4), db + (uint64_t)((k * UK) >> 4), idesc,
                               (kb != kb0 || k != 0) ? 1u : 0u);
                    mma_commit(&ctl->empty[s]);
                }
                if (!ok) break;
                mma_commit(&ctl->tfull[acc]);
                acc ^= 1u;
                if (acc == 0) acc_ph ^= 1u;
            }
            // Every MMA this thread issued has retired once `drained` fires
            // (waited on with a private flag: an abort raised elsewhere must
            // not skip the drain before TMEM is released).
            mma_commit(&ctl->drained);
            volatile int never = 0;
            mbar_wait(&ctl->drained, 0, &never, 200000000ull);
        }
    } else if (warp < 2 + kEpiWarps) {
        // ---------------- epilogue (warps 2..9) ----------------
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;       // which 32-column blocks of the tile it takes
        // With BN = 32 a tile has one column block: the two halves take
        // alternate tiles instead (the tiles of accumulator 0, of 1), so two
        // tiles drain at once; the other half only releases the accumulator.
        uint32_t acc = 0, acc_ph = 0;
        bool row_accum = false;
        if constexpr (HasRowAccum<Epi>::value && BN == 32) row_accum = n_tiles == 1 && sh.splits == 1;
        if constexpr (HasRowAccum<Epi>::value && BN == 32) {
            if (row_accum) {
                // N <= 16: the halves take alternate tiles, columns [0, 16).
                // N > 16: both halves take every tile, half h columns [16 h, +16).
                const bool alt = N <= 16;
                const int c0 = alt ? 0 : 16 * half;
                typename Epi::Accum st;
                epi.acc_init(st);
                for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
                    int m0, n0, kb0, kb1;
                    tile_coords(t, m0, n0, kb0, kb1);
                    const bool ok = mbar_wait(&ctl->tfull[acc], acc_ph, abort);
                    __syncwarp();
                    if (!__all_sync(0xffffffffu, ok)) break;
                    tc_fence_after();
                    const bool mine = !alt || (int)acc == half;
                    if (mine && c0 < N && kb0 < kb1) {
                        uint32_t v[32];
                        tmem_ld_32x32b_x32(tbase + ((uint32_t)(q * 32) << 16) + acc * BN, v);
                        tmem_ld_wait();
                        epi.store_acc(m0 + q * 32 + lane, c0, M, N, v, c0 != 0, st);
                    }
                    tc_fence_before();
                    __syncwarp();  // every lane's TMEM reads are done: one arrival per warp
                    if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
                    acc ^= 1u;
                    if (acc == 0) acc_ph ^= 1u;
                }
                __syncwarp();
                epi.acc_flush(st, c0, N, lane, epi_sm);
            }
        }
        for (int t = blockIdx.x; t < tiles && !row_accum; t += gridDim.x) {
            int m0, n0, kb0, kb1;
            tile_coords(t, m0, n0, kb0, kb1);
            const bool ok = mbar_wait(&ctl->tfull[acc], acc_ph, abort);
            __syncwarp();  // reconverge before the warp-collective tcgen05.ld
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = m0 + q * 32 + lane;
            const bool empty_split = kb0 >= kb1;  // nothing accumulated: skip
            const bool mine = BN > 32 || (int)acc == half;
#pragma unroll 1
            for (int c0 = BN > 32 ? 32 * half : 0; mine && c0 < BN && n0 + c0 < N && !empty_split;
                 c0 += (BN > 32 ? 64 : 32)) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + ((uint32_t)(q * 32) << 16) + acc * BN + c0, v);
                tmem_ld_wait();
                epi.store(row, n0 + c0, M, N, v, lane, epi_sm);
            }
            tc_fence_before();
            __syncwarp();  // every lane's TMEM reads are done: one arrival per warp
            if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
            acc ^= 1u;
            if (acc == 0) acc_ph ^= 1u;
        }
    } else if constexpr (Src::kGather) {
        // ---------------- implicit-GEMM producers (warps 10..) ----------------
        // Thread g copies 16-byte piece (g & 7) of rows (g >> 3) + kRowStep i
        // of every stage: eight consecutive threads fill one 128-byte row.
        constexpr int kRowStep = 32 * kGatherWarps / 8, kRowsPer = BM / kRowStep;
        const int g = threadIdx.x - 32 * (2 + kEpiWarps);
        const int l8 = g & 7, rs = g >> 3;
        const int cmask = (1 << src.lgC) - 1, ntaps = src.kh * src.kw;
        uint32_t it = 0;
        for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
            int m0, n0, kb0, kb1;
            tile_coords(t, m0, n0, kb0, kb1);
            int iy0[kRowsPer], ix0[kRowsPer], pb[kRowsPer];  // the rows' top-left input tap, b * H (-1: no row)
#pragma unroll
            for (int i = 0; i < kRowsPer; ++i) {
                const int m = m0 + rs + kRowStep * i;
                const int b = m / src.HoWo, p = m - b * src.HoWo, oy = p / src.Wo, ox = p - oy * src.Wo;
                iy0[i] = oy * src.sh - src.ph;
                ix0[i] = ox * src.sw - src.pw;
                pb[i] = m < M ? b * src.H : -1;
            }
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int s = it % G::STAGES;
                const uint32_t ph = (it / G::STAGES) & 1u;
                if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort)) break;
                const int koff = kb * BK + l8 * 16;
                const int tap = koff >> src.lgC, ci0 = koff & cmask;
                const bool tok = tap < ntaps;
                const int ky = tok ? tap / src.kw : 0, kx = tok ? tap - ky * src.kw : 0;
                uint8_t *stage = sA + s * G::A_BYTES;
#pragma unroll
                for (int i = 0; i < kRowsPer; ++i) {
                    const int r = rs + kRowStep * i;
                    const int iy = iy0[i] + ky, ix = ix0[i] + kx;
                    const bool ok = tok && pb[i] >= 0 && (unsigned)iy < (unsigned)src.H && (unsigned)ix < (unsigned)src.W;
                    const int8_t *gp = ok ? src.x + ((((i64)(pb[i] + iy) * src.W + ix) << src.lgC) + ci0) : src.x;
                    cp_async16(stage + r * BK + ((l8 ^ (r & 7)) << 4), gp, ok ? 16u : 0u);
                }
                // arrives on the stage's A barrier once these copies have landed
                cp_async_arrive_noinc(&ctl->afull[s]);
            }
        }
        cp_async_wait<0>();  // nothing may land after the CTA is gone
    }

    __syncthreads();
    if (warp >= 2) epi.finish(epi_sm, N);
    if (threadIdx.x == 0 && *abort) {
        // Drain loads that were issued but never waited for, so no TMA write
        // lands in shared memory after the CTA is gone (bounded as well).
        for (uint32_t i = ctl->consumed; i < ctl->issued; ++i) {
            volatile int never = 0;
            mbar_wait(&ctl->full[i % G::STAGES], (i / G::STAGES) & 1u, &never, 200000000ull);
        }
        atomicExch(&g_tc_error, 1);
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, G::TMEM_COLS);
    }
}

// ------------------------------------------------- CTA-pair (2-SM) variant
// For large M x N (at least one wave of 256 x 256 tiles): a cluster of two
// CTAs computes one 256 x 256 tile with tcgen05.mma.cta_group::2.  CTA r
// loads rows [m0 + 128 r, +128) of A and rows [n0 + 128 r, +128) of B (its
// half of the tile's B) into its own shared memory; CTA 0 issues M = 256 MMAs
// that read both halves and write 128 accumulator rows into each CTA's TMEM.
// Per SM a 128-byte K slice costs 32 KB of operand traffic instead of the
// single-CTA 48 KB for the same multiply-adds, and six stages fit.
//   full[s]   (CTA 0): armed by CTA 0 with both CTAs' bytes, completed by
//             the TMA loads of both CTAs.
//   empty[s]  (each CTA): released by CTA 0's MMA commit (one commit per CTA).
//   tfull[a]  (each CTA): accumulator a is ready (commits as above).
//   tempty[a] (CTA 0): released by the epilogue warps of both CTAs (one
//             arrival per warp, after the warp's TMEM reads).
// All waits are bounded as in the single-CTA kernel; the CTAs meet at a
// cluster barrier before TMEM is freed.
constexpr int kPairBN = 256;   // N of one pair MMA; each CTA holds 128 rows of B
constexpr int kPairStages = 6;
// Epilogue warps of the pair kernel: 16 (four per TMEM lane quarter) for the
// arithmetic epilogues, 8 for the plain s32 store and the s32 atomics, which
// are bound by their stores (more warps measured slower there) and stage
// 1 KB per warp in the epilogue scratch.
template <class Epi>
constexpr int pair_epi_warps() {
    return std::is_same<Epi, EpiS32>::value || std::is_same<Epi, EpiS32Atomic>::value ? 8 : 16;
}

struct PairCfg {
    static constexpr int A_BYTES = BM * BK;               // 16 KB
    static constexpr int B_BYTES = (kPairBN / 2) * BK;    // 16 KB
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * kPairBN;         // two accumulators: the whole TMEM
    // per-column sums (2 x kMaxN doubles), or 1 KB of store staging per
    // epilogue warp (16 warps)
    static constexpr int EPI_SMEM = 2 * kMaxN * 8 > 16 * 1024 ? 2 * kMaxN * 8 : 16 * 1024;
    static constexpr int SMEM = 1024 + kPairStages * STAGE_BYTES + 512 + EPI_SMEM;
};

template <class Epi, int EW = pair_epi_warps<Epi>()>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Shape sh,
                    Epi epi) {
    using G = PairCfg;
    static_assert(EW * 1024 <= G::EPI_SMEM, "the store epilogues stage 1 KB per epilogue warp");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + kPairStages * G::A_BYTES;
    Ctl *ctl = reinterpret_cast<Ctl *>(smem + kPairStages * G::STAGE_BYTES);
    double *epi_sm = reinterpret_cast<double *>(smem + kPairStages * G::STAGE_BYTES + 512);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int M = sh.M, N = sh.N, K = sh.K;
    const int m_tiles = (M + 2 * BM - 1) / (2 * BM), n_tiles = (N + kPairBN - 1) / kPairBN;
    const int tiles = m_tiles * n_tiles, kblocks = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&ctl->tfull[a], 1);
            mbar_init(&ctl->tempty[a], 2 * EW);  // one arrival per epilogue warp of either CTA
        }
        mbar_init(&ctl->drained, 1);
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp >= 2) epi.init(epi_sm);
    if (warp == 1) {
        tmem_alloc_pair(&ctl->tmem_base, G::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // barriers of both CTAs initialised before any remote use
    tc_fence_after();
    const uint32_t tbase = ctl->tmem_base;
    volatile int *abort = &ctl->abort;

    auto tile_coords = [&](int t, int &m0, int &n0) {
        m0 = (t / n_tiles) * (2 * BM);
        n0 = (t % n_tiles) * kPairBN;
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            uint32_t it = 0;
            for (int t = pair; t < tiles && !*abort; t += npairs) {
                int m0, n0;
                tile_coords(t, m0, n0);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    const uint32_t ph = (it / kPairStages) & 1u;
                    if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort)) break;
                    if (rank == 0) mbar_expect_tx(&ctl->full[s], 2 * G::STAGE_BYTES);
                    const uint32_t full0 = mapa_shared(smem_u32(&ctl->full[s]), 0);
                    tma_load_2d_pair(sA + s * G::A_BYTES, &tmA, full0, kb * BK, m0 + (int)rank * BM);
                    tma_load_2d_pair(sB + s * G::B_BYTES, &tmB, full0, kb * BK, n0 + (int)rank * (kPairBN / 2));
                    ctl->issued = it + 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (CTA 0) ----------------
            constexpr uint32_t idesc = idesc_i8(2 * BM, kPairBN);
            uint32_t it = 0, acc = 0, acc_ph = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                if (!(ok = mbar_wait(&ctl->tempty[acc], acc_ph ^ 1u, abort))) break;
                tc_fence_after();
                const uint32_t d = tbase + acc * kPairBN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    const uint32_t ph = (it / kPairStages) & 1u;
                    if (!(ok = mbar_wait(&ctl->full[s], ph, abort))) break;
                    ctl->consumed = it + 1;
                    tc_fence_after();
                    const uint64_t da = desc_k_sw128(smem_u32(sA + s * G::A_BYTES));
                    const uint64_t db = desc_k_sw128(smem_u32(sB + s * G::B_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / UK; ++k)
                        mma_i8_pair(d, da + (uint64_t)((k * UK) >> 4), db + (uint64_t)((k * UK) >> 4), idesc,
                                    (kb != 0 || k != 0) ? 1u : 0u);
                    const uint32_t e_loc = smem_u32(&ctl->empty[s]);
                    mma_commit_pair(e_loc);
                    mma_commit_pair(mapa_shared(e_loc, 1));
                }
                if (!ok) break;
                const uint32_t f_loc = smem_u32(&ctl->tfull[acc]);
                mma_commit_pair(f_loc);
                mma_commit_pair(mapa_shared(f_loc, 1));
                acc ^= 1u;
                if (acc == 0) acc_ph ^= 1u;
            }
            mma_commit_pair(smem_u32(&ctl->drained));
            volatile int never = 0;
            mbar_wait(&ctl->drained, 0, &never, 200000000ull);
        }
    } else {
        // ---------------- epilogue (warps 2..EW+1, both CTAs) ----------------
        const int q = warp & 3;
        const int grp = (warp - 2) >> 2;  // column group: blocks 32 * grp, 32 * grp + 8 * EW, ...
        uint32_t acc = 0, acc_ph = 0;
        for (int t = pair; t < tiles; t += npairs) {
            int m0, n0;
            tile_coords(t, m0, n0);
            const bool ok = mbar_wait(&ctl->tfull[acc], acc_ph, abort);
            __syncwarp();
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = m0 + (int)rank * BM + q * 32 + lane;
#pragma unroll 1
            for (int c0 = 32 * grp; c0 < kPairBN && n0 + c0 < N; c0 += 8 * EW) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + ((uint32_t)(q * 32) << 16) + acc * kPairBN + c0, v);
                tmem_ld_wait();
                epi.store(row, n0 + c0, M, N, v, lane, epi_sm);
            }
            tc_fence_before();
            __syncwarp();  // every lane's TMEM reads are done: one (remote) arrival per warp
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->tempty[acc]), 0));
            acc ^= 1u;
            if (acc == 0) acc_ph ^= 1u;
        }
    }

    __syncthreads();
    if (warp >= 2) epi.finish(epi_sm, N);
    if (threadIdx.x == 0 && *abort) {
        if (rank == 0) {
            for (uint32_t i = ctl->consumed; i < ctl->issued; ++i) {
                volatile int never = 0;
                mbar_wait(&ctl->full[i % kPairStages], (i / kPairStages) & 1u, &never, 200000000ull);
            }
        }
        atomicExch(&g_tc_error, 1);
    }
    __syncthreads();
    cluster_sync();  // the peer has finished with this CTA's barriers and TMEM
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tbase, G::TMEM_COLS);
    }
}


// Every s32 accumulator value a (as the float the epilogue converts it to)
// through the FMA division and the IEEE division by b: counts the results
// that differ in any bit.
__global__ void division_check_kernel(float b, float r, unsigned long long *bad) {
    unsigned long long local = 0;
    const long long n = 1ll << 32, stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float a = (float)(int32_t)(uint32_t)i;
        if (__float_as_uint(div_by(a, b, r)) != __float_as_uint(__fdiv_rn(a, b))) ++local;
    }
    if (local) atomicAdd(bad, local);
}

// CUDA-core fallback for operands TMA cannot describe (base address not
// 16-byte aligned): 64x64 tile per CTA, K in 32-byte slices, dp4a.
__global__ void gemm_i8_simt_kernel(const int8_t *__restrict__ A, const int8_t *__restrict__ B,
                                    int32_t *__restrict__ C, int M, int N, int K, int ld) {
    __shared__ int32_t sa[64][9];  // 32 bytes of K per row packed as 8 words (+1 pad)
    __shared__ int32_t sb[64][9];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads, 4x4 outputs each
    const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
    int acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int e = threadIdx.x; e < 64 * 8; e += 256) {
            const int r = e >> 3, w = e & 7;
            uint32_t pa = 0, pb = 0;
            for (int b = 0; b < 4; ++b) {
                const int k = k0 + w * 4 + b;
                const uint8_t va = (m0 + r < M && k < K) ? (uint8_t)A[(i64)(m0 + r) * ld + k] : 0;
                const uint8_t vb = (n0 + r < N && k < K) ? (uint8_t)B[(i64)(n0 + r) * ld + k] : 0;
                pa |= (uint32_t)va << (8 * b);
                pb |= (uint32_t)vb << (8 * b);
            }
            sa[r][w] = (int32_t)pa;
            sb[r][w] = (int32_t)pb;
        }
        __syncthreads();
#pragma unroll
        for (int w = 0; w < 8; ++w)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __dp4a(sa[ty * 4 + i][w], sb[tx * 4 + j][w], acc[i][j]);
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            const int r = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
            if (r < M && c < N) C[(i64)r * N + c] = acc[i][j];
        }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

template <int BN, class Epi, class Src = TmaA>
void launch_tc(const CUtensorMap &ta, const CUtensorMap &tb, Shape sh, const Epi &epi, cudaStream_t st,
               const Src &src = Src()) {
    using G = Cfg<BN>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        TRBA_CHECK(cudaFuncSetAttribute(gemm_i8_tc_kernel<BN, Epi, Src>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
        attr_set[dev] = true;
    }
    const int tiles = ((sh.M + BM - 1) / BM) * ((sh.N + BN - 1) / BN) * sh.splits;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_i8_tc_kernel<BN, Epi, Src><<<grid, threads_for<Src>(), G::SMEM, st>>>(ta, tb, sh, epi, src);
    TRBA_LAUNCH_CHECK();
}

int g_pair_enabled = 1;  // host-side switch (trba_gemm_pair_enable)
bool pair_enabled() { return g_pair_enabled != 0; }

// The pair kernel serves unsplit problems with N a multiple of 256 and at
// least one wave of pair tiles; everything else takes the single-CTA kernel.
bool use_pair(const Shape &sh) {
    if (sh.splits != 1 || sh.N < kPairBN || (sh.N % kPairBN) != 0) return false;
    const int tiles = ((sh.M + 2 * BM - 1) / (2 * BM)) * (sh.N / kPairBN);
    return tiles >= sm_count() / 2;
}

template <class Epi>
void launch_pair(const CUtensorMap &ta, const CUtensorMap &tb, Shape sh, const Epi &epi, cudaStream_t st) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        TRBA_CHECK(cudaFuncSetAttribute(gemm_i8_pair_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        PairCfg::SMEM));
        attr_set[dev] = true;
    }
    const int tiles = ((sh.M + 2 * BM - 1) / (2 * BM)) * (sh.N / kPairBN);
    const int pairs = tiles < sm_count() / 2 ? tiles : sm_count() / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3(64 + 32 * pair_epi_warps<Epi>());
    cfg.dynamicSmemBytes = PairCfg::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TRBA_CHECK(cudaLaunchKernelEx(&cfg, gemm_i8_pair_kernel<Epi>, ta, tb, sh, epi));
    TRBA_LAUNCH_CHECK();
}

template <class Epi>
bool run_tc(const int8_t *A, int lda, const int8_t *B, int ldb, Shape sh, const Epi &epi, cudaStream_t st) {
    if (use_pair(sh) && pair_enabled()) {
        CUtensorMap ta, tb;
        if (make_tmap_i8(&ta, A, sh.M, sh.K, lda, BM) && make_tmap_i8(&tb, B, sh.N, sh.K, ldb, kPairBN / 2)) {
            launch_pair(ta, tb, sh, epi, st);
            return true;
        }
    }
    const int bn = pick_bn(sh.N);
    CUtensorMap ta, tb;
    if (!make_tmap_i8(&ta, A, sh.M, sh.K, lda, BM) || !make_tmap_i8(&tb, B, sh.N, sh.K, ldb, bn)) return false;
    switch (bn) {
        case 32: launch_tc<32>(ta, tb, sh, epi, st); break;
        case 64: launch_tc<64>(ta, tb, sh, epi, st); break;
        case 128: launch_tc<128>(ta, tb, sh, epi, st); break;
        default: launch_tc<256>(ta, tb, sh, epi, st); break;
    }
    return true;
}

// The implicit-GEMM conv forward (ConvGather): B = the weights in the
// gather's K order, [N, kh*kw*Cin] with leading dimension ldw.
template <class Epi>
bool run_conv_gather(const ConvGeo &g, const int8_t *Wh, int ldw, int N, const Epi &epi, cudaStream_t st) {
    if (!conv_implicit_ok(g)) return false;
    const int K = g.kh * g.kw * g.Cin, M = g.B * g.Ho * g.Wo;
    const int bn = pick_bn(N);
    CUtensorMap tb;
    if (!make_tmap_i8(&tb, Wh, N, K, ldw, bn)) return false;
    int lg = 0;
    while ((1 << lg) < g.Cin) ++lg;
    const ConvGather src{g.x, g.H, g.W, lg, g.kh, g.kw, g.sh, g.sw, g.ph, g.pw, g.Wo, g.Ho * g.Wo};
    const int kblocks = (K + BK - 1) / BK;
    const Shape sh{M, N, K, 1, kblocks};
    switch (bn) {
        case 32: launch_tc<32>(tb, tb, sh, epi, st, src); break;
        case 64: launch_tc<64>(tb, tb, sh, epi, st, src); break;
        case 128: launch_tc<128>(tb, tb, sh, epi, st, src); break;
        default: launch_tc<256>(tb, tb, sh, epi, st, src); break;
    }
    return true;
}

Shape make_shape(int M, int N, int K, int splits) {
    const int kblocks = (K + BK - 1) / BK;
    if (splits < 1) splits = 1;
    if (splits > kblocks) splits = kblocks;
    const int per = (kblocks + splits - 1) / splits;
    return Shape{M, N, K, (kblocks + per - 1) / per, per};
}

}  // namespace

namespace trba {

bool make_tmap_i8(CUtensorMap *m, const void *ptr, int rows, int k, int ld, int box_rows) {
    auto enc = encode_fn();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld & 15) || ld < k) return false;
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int pick_bn(int N) { return N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256; }

bool gemm_i8_tc(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld, cudaStream_t st) {
    EpiS32 e{C, N, ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && (N & 3) == 0};
    return run_tc(A, ld, B, ld, make_shape(M, N, K, 1), e, st);
}

bool gemm_i8_splitk_atomic(const int8_t *A, int lda, const int8_t *B, int ldb, int32_t *C, int M, int N, int K,
                           int splits, cudaStream_t st) {
    return run_tc(A, lda, B, ldb, make_shape(M, N, K, splits), EpiS32Atomic{C, N}, st);
}

bool gemm_i8_conv_f32(const int8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, float *x,
                      const float *s_in, const float *w_s, bool per_channel, double *bn_acc, int HW, cudaStream_t st) {
    if (N > kMaxN) return false;
    return run_tc(A, lda, B, ldb, make_shape(M, N, K, 1), EpiConvF32{x, s_in, w_s, per_channel ? 1 : 0, bn_acc, HW},
                  st);
}

// RN(1 / d) (the float nearest 1/d: no ties exist) when d is in the range of
// the FMA division path (2^-90 <= |d| <= 2^90), else false.
bool division_reciprocal(float d, float &r) {
    if (!std::isfinite(d)) return false;
    const float ad = std::fabs(d);
    if (!(ad >= 0x1p-90f && ad <= 0x1p90f)) return false;
    // (float)(1.0 / d) may round twice (to double, then to float): keep the
    // float among it and its two neighbours with the smallest |f d - 1|,
    // which double evaluates exactly (24 + 24 significand bits).
    const float c = (float)(1.0 / (double)d);
    float best = c;
    double err = std::fabs((double)c * (double)d - 1.0);
    for (const float f : {std::nextafter(c, -INFINITY), std::nextafter(c, INFINITY)}) {
        const double e = std::fabs((double)f * (double)d - 1.0);
        if (e < err) best = f, err = e;
    }
    r = best;
    return true;
}

bool gemm_i8_requant(const int8_t *A, const int8_t *B, int8_t *out, const float *bias, int M, int N, int K, int ld,
                     float div, float mul, cudaStream_t st) {
    EpiRequantI8 e{out, N, bias, div, mul, ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && (N & 15) == 0, 0.0f,
                   false};
    e.fast_div = division_reciprocal(div, e.rdiv);
    return run_tc(A, ld, B, ld, make_shape(M, N, K, 1), e, st);
}

bool gemm_i8_dequant(const int8_t *A, const int8_t *B, float *out, const float *w_scale, float a_scale,
                     const float *bias, int relu, int M, int N, int K, int ld, cudaStream_t st) {
    EpiDequantF32 e{out, N, w_scale, bias, a_scale, relu,
                    ((reinterpret_cast<uintptr_t>(out) & 15) == 0) && (N & 3) == 0};
    return run_tc(A, ld, B, ld, make_shape(M, N, K, 1), e, st);
}

bool conv_implicit_ok(const ConvGeo &g) {
    const bool pow2 = g.Cin >= 16 && g.Cin <= 1024 && (g.Cin & (g.Cin - 1)) == 0;
    return pow2 && (reinterpret_cast<uintptr_t>(g.x) & 15) == 0 && g.B > 0 && g.Ho > 0 && g.Wo > 0 &&
           (i64)g.B * g.Ho * g.Wo < (1ll << 31) && (i64)g.B * g.H * g.W * g.Cin < (1ll << 40);
}

bool gemm_i8_conv_implicit_f32(const ConvGeo &g, const int8_t *Wh, int ldw, int N, float *x, const float *s_in,
                               const float *w_s, bool per_channel, double *bn_acc, cudaStream_t st) {
    if (N > kMaxN) return false;
    return run_conv_gather(g, Wh, ldw, N, EpiConvF32{x, s_in, w_s, per_channel ? 1 : 0, bn_acc, g.Ho * g.Wo}, st);
}

bool gemm_i8_conv_implicit_s32(const ConvGeo &g, const int8_t *Wh, int ldw, int N, int32_t *C, cudaStream_t st) {
    EpiS32 e{C, N, ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && (N & 3) == 0};
    return run_conv_gather(g, Wh, ldw, N, e, st);
}

int splitk_for(int M, int N, int K) {
    // Enough (m, n, split) tiles for two waves of SMs, at least 2 K blocks each.
    const int tiles = ((M + BM - 1) / BM) * ((N + 127) / 128);
    const int kblocks = (K + BK - 1) / BK;
    int s = (2 * sm_count() + tiles - 1) / tiles;
    if (s > kblocks / 2) s = kblocks / 2;
    return s < 1 ? 1 : s;
}

void gemm_i8_simt(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld, cudaStream_t st) {
    dim3 grid((M + 63) / 64, (N + 63) / 64);
    gemm_i8_simt_kernel<<<grid, 256, 0, st>>>(A, B, C, M, N, K, ld);
    TRBA_LAUNCH_CHECK();
}

}  // namespace trba

extern "C" {

void launch_gemm_int8(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    const int ld = (k + 15) & ~15;
    if (!gemm_i8_tc(a, b, c, m, n, k, ld, as_stream(stream))) gemm_i8_simt(a, b, c, m, n, k, ld, as_stream(stream));
}

// Test hook: route the same call through the CUDA-core kernel.
void trba_gemm_int8_simt(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    gemm_i8_simt(a, b, c, m, n, k, (k + 15) & ~15, as_stream(stream));
}

// Split-K variant: C (zeroed by the caller) += A . Bt^T, K split `splits`
// ways (0 = automatic), partial tiles combined with integer atomics.
void trba_gemm_int8_splitk(const int8_t *a, const int8_t *b, int32_t *c, int m, int n, int k, int splits,
                           void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    const int ld = (k + 15) & ~15;
    if (splits <= 0) splits = splitk_for(m, n, k);
    if (!gemm_i8_splitk_atomic(a, ld, b, ld, c, m, n, k, splits, as_stream(stream)))
        report_error(__FILE__, __LINE__, "trba_gemm_int8_splitk: operands not 16-byte aligned", -1);
}

// GEMM + the conv inference epilogue in one kernel: out int8 [m, n] =
// launch_gemm_int8 followed by launch_conv_epilogue(acc, bias, out, n, div,
// mul, m, n, 1, 1).  Operands as launch_gemm_int8 (padded, 16-byte aligned).
void trba_gemm_int8_requant(const int8_t *a, const int8_t *b, const float *bias, int8_t *out, int m, int n, int k,
                            float acc_div, float out_mul, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    const int ld = (k + 15) & ~15;
    if (gemm_i8_requant(a, b, out, bias, m, n, k, ld, acc_div, out_mul, as_stream(stream))) return;
    int32_t *acc = nullptr;
    TRBA_CHECK(cudaMallocAsync((void **)&acc, (size_t)m * n * sizeof(int32_t), as_stream(stream)));
    if (!acc) return;
    gemm_i8_simt(a, b, acc, m, n, k, ld, as_stream(stream));
    launch_conv_epilogue(acc, bias, out, n, acc_div, out_mul, m, n, 1, 1, stream);
    TRBA_CHECK(cudaFreeAsync(acc, as_stream(stream)));
}

// GEMM + per-channel dequantisation (+ bias, + ReLU) in one kernel:
// out f32 [m, n] = act((float)acc * (a_scale * w_scale[n]) [+ bias[n]]).
void trba_gemm_int8_dequant_f32(const int8_t *a, const int8_t *b, const float *w_scale, float a_scale,
                                const float *bias, int relu, float *out, int m, int n, int k, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return;
    TRBA_REQUIRE(w_scale != nullptr, "trba_gemm_int8_dequant_f32: w_scale is required");
    const int ld = (k + 15) & ~15;
    if (gemm_i8_dequant(a, b, out, w_scale, a_scale, bias, relu, m, n, k, ld, as_stream(stream))) return;
    report_error(__FILE__, __LINE__, "trba_gemm_int8_dequant_f32: operands not 16-byte aligned", -1);
}

// The requant epilogue's division against the IEEE division for all 2^32
// s32 accumulator values and one divisor (synchronous): the number of
// results that differ, or -1 when the divisor is outside the FMA path's
// range (the epilogue then divides with the IEEE division itself).
long long trba_requant_division_check(float div, void *stream) {
    float r = 0.0f;
    if (!division_reciprocal(div, r)) return -1;
    cudaStream_t st = as_stream(stream);
    unsigned long long *bad = nullptr, h = 0;
    TRBA_CHECK(cudaMallocAsync((void **)&bad, sizeof(unsigned long long), st));
    if (!bad) return -2;
    TRBA_CHECK(cudaMemsetAsync(bad, 0, sizeof(unsigned long long), st));
    division_check_kernel<<<sm_count() * 8, 256, 0, st>>>(div, r, bad);
    TRBA_LAUNCH_CHECK();
    TRBA_CHECK(cudaMemcpyAsync(&h, bad, sizeof(h), cudaMemcpyDeviceToHost, st));
    TRBA_CHECK(cudaStreamSynchronize(st));
    TRBA_CHECK(cudaFreeAsync(bad, st));
    return (long long)h;
}

// Device-side error word of the tensor-core kernels (1 = a bounded wait
// timed out).  Synchronises the device; clears the word when `clear` != 0.
int trba_tc_error_poll(int clear) {
    int v = 0;
    TRBA_CHECK(cudaDeviceSynchronize());
    TRBA_CHECK(cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)));
    if (clear) {
        const int z = 0;
        TRBA_CHECK(cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int)));
    }
    // the input-gradient kernel keeps its own word (another translation unit)
    return (v | trba::dgtc::error_poll(clear != 0)) ? 1 : 0;
}

}  // extern "C"

extern "C" int trba_gemm_pair_enable(int enable) {
    const int prev = g_pair_enabled;
    g_pair_enabled = enable ? 1 : 0;
    return prev;
}
