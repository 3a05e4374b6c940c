// launch_gemm_int8 on B200: C[M,N] s32 = A[M,K] . Bt[N,K]^T with tcgen05
// kind::i8 tensor cores (reference contract: cuda/kernels.cu:227-250 of the
// checked-out tree, operands row-major with leading dimension align16(K)).
//
// Design (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0 lane 0 : TMA producer. For each 128 x BN output tile it streams
//                   128-byte K slices of A (128 rows) and B (BN rows) into a
//                   STAGES-deep ring of 128B-swizzled shared-memory stages.
//   warp 1 lane 0 : MMA issuer. Four tcgen05.mma (M=128, N=BN, K=32) per
//                   stage into one of two TMEM accumulators, so the epilogue
//                   of tile i overlaps the MMAs of tile i+1.
//   warps 2..5    : epilogue. tcgen05.ld 32 columns at a time (each thread
//                   owns one output row) and stores s32 to global memory.
// Tensor maps cover exactly [M, K] and [N, K]: TMA zero-fills every
// out-of-range row and column, so the kernel never reads the operands'
// padding and needs no tail handling in the main loop.
//
// Every mbarrier wait is bounded (2 s): on a timeout the CTA raises an abort
// flag, every role leaves its loop, in-flight loads are drained, TMEM is
// freed and the device error word g_tc_error is set for the host to read.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "gemm_i8.cuh"
#include "tc_primitives.cuh"

using namespace trba;
using namespace trba::tc;

__device__ int g_tc_error = 0;

namespace {

constexpr int BM = 128;   // UMMA M (cta_group::1)
constexpr int BK = 128;   // bytes of K per stage = one 128B swizzle row
constexpr int UK = 32;    // K of one kind::i8 MMA
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // two accumulators (power of two >= 64)
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 512;
};

struct Ctl {  // lives after the stage ring in shared memory
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drained;
    uint32_t tmem_base;
    int abort;
    uint32_t issued;    // stage loads issued by the producer
    uint32_t consumed;  // stage loads whose data the MMA warp waited for
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  int M, int N, int K, int32_t *__restrict__ C) {
    using G = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + G::STAGES * G::A_BYTES;
    Ctl *ctl = reinterpret_cast<Ctl *>(smem + G::STAGES * G::STAGE_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles, kblocks = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&ctl->tfull[a], 1);
            mbar_init(&ctl->tempty[a], 4 * 32);
        }
        mbar_init(&ctl->drained, 1);
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(&ctl->tmem_base, G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = ctl->tmem_base;
    volatile int *abort = &ctl->abort;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t it = 0;
            for (int t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
                const int m0 = (t / n_tiles) * BM, n0 = (t % n_tiles) * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % G::STAGES;
                    const uint32_t ph = (it / G::STAGES) & 1u;
                    if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort)) break;
                    mbar_expect_tx(&ctl->full[s], G::STAGE_BYTES);
                    tma_load_2d(sA + s * G::A_BYTES, &tmA, &ctl->full[s], kb * BK, m0);
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
                if (!(ok = mbar_wait(&ctl->tempty[acc], acc_ph ^ 1u, abort))) break;
                tc_fence_after();
                const uint32_t d = tbase + acc * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % G::STAGES;
                    const uint32_t ph = (it / G::STAGES) & 1u;
                    if (!(ok = mbar_wait(&ctl->full[s], ph, abort))) break;
                    ctl->consumed = it + 1;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * G::A_BYTES), b0 = smem_u32(sB + s * G::B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / UK; ++k)
                        mma_i8(d, desc_k_sw128(a0 + k * UK), desc_k_sw128(b0 + k * UK), idesc,
                               (kb | k) != 0);
                    mma_commit(&ctl->empty[s]);
                }
                if (!ok) break;
                mma_commit(&ctl->tfull[acc]);
                acc ^= 1u;
                if (acc == 0) acc_ph ^= 1u;
            }
            // Every MMA this thread issued has retired once `drained` fires.
            // (waited on with a private flag: an abort raised elsewhere must
            // not skip the drain before TMEM is released)
            mma_commit(&ctl->drained);
            volatile int never = 0;
            mbar_wait(&ctl->drained, 0, &never, 200000000ull);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint32_t acc = 0, acc_ph = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const bool ok = mbar_wait(&ctl->tfull[acc], acc_ph, abort);
            __syncwarp();  // reconverge before the warp-collective tcgen05.ld
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int m0 = (t / n_tiles) * BM, n0 = (t % n_tiles) * BN;
            const int row = m0 + q * 32 + lane;
            int32_t *crow = C + (i64)row * N;
#pragma unroll 1
            for (int c0 = 0; c0 < BN && n0 + c0 < N; c0 += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + ((uint32_t)(q * 32) << 16) + acc * BN + c0, v);
                tmem_ld_wait();
                if (row < M) {
                    const int col = n0 + c0;
                    if (col + 32 <= N && (N & 3) == 0) {
                        int4 *dst = reinterpret_cast<int4 *>(crow + col);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            dst[j] = make_int4((int)v[4 * j], (int)v[4 * j + 1], (int)v[4 * j + 2], (int)v[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col + j < N) crow[col + j] = (int32_t)v[j];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&ctl->tempty[acc]);
            acc ^= 1u;
            if (acc == 0) acc_ph ^= 1u;
        }
    }

    __syncthreads();
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

template <int BN>
void launch_tc(const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K, int32_t *C,
               cudaStream_t st) {
    using G = Cfg<BN>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        TRBA_CHECK(cudaFuncSetAttribute(gemm_i8_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
        attr_set[dev] = true;
    }
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_i8_tc_kernel<BN><<<grid, kThreads, G::SMEM, st>>>(ta, tb, M, N, K, C);
    TRBA_LAUNCH_CHECK();
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

// Returns false when the operands cannot be described by a tensor map (the
// caller then uses the CUDA-core kernel).
bool gemm_i8_tc(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld,
                cudaStream_t st) {
    const int bn = pick_bn(N);
    CUtensorMap ta, tb;
    if (!make_tmap_i8(&ta, A, M, K, ld, BM) || !make_tmap_i8(&tb, B, N, K, ld, bn)) return false;
    switch (bn) {
        case 32: launch_tc<32>(ta, tb, M, N, K, C, st); break;
        case 64: launch_tc<64>(ta, tb, M, N, K, C, st); break;
        case 128: launch_tc<128>(ta, tb, M, N, K, C, st); break;
        default: launch_tc<256>(ta, tb, M, N, K, C, st); break;
    }
    return true;
}

void gemm_i8_simt(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K, int ld,
                  cudaStream_t st) {
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
    return v;
}

}  // extern "C"
