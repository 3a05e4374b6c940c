// Sequence head of the device-resident QAT step: fp32 GEMM, BiLSTM time
// loops, attention decoder, CE and CTC.  The recurrences are latency-bound
// (T <= 64 dependent steps over tiny matrices), so each runs as ONE
// persistent launch per direction / decoder with the recurrent weights in
// shared memory and one CTA per group of samples (samples never interact
// inside a recurrence); the big batched products (input projections, weight
// gradients, logits) run as ordinary GEMMs outside the time loop.
#include <atomic>
#include "seq_kernels.cuh"

namespace trba {
namespace seq {
namespace {

__device__ __forceinline__ float sigm(float v) { return cr_sigmoid(v); }

// ------------------------------------------------------------- sgemm --
constexpr int TM = 64, TN = 64, TK = 16;

__device__ __forceinline__ void gemm_store(const Gemm &g, int m, int n, double acc) {
    float v = (float)acc;
    float *c = g.C + (i64)m * g.ldc + n;
    if (g.accumulate) v = fadd(v, *c);
    if (g.bias) v = fadd(v, g.bias[n]);
    *c = v;
}

// One 64x64 output tile over the K range of split blockIdx.z (f64
// accumulation, products of f32 operands are exact in f64).  The operand
// tiles are converted to f64 once, when staged in shared memory; the loader
// walks the operand's unit-stride dimension with consecutive threads so the
// global reads coalesce whichever way the operand is laid out, and the next
// K tile is read into registers while the current one is multiplied.  Thread
// (tx, ty) owns rows ty + 16 i and columns tx + 16 j (i, j < 4), so a warp's
// shared-memory reads are broadcasts (A) or 16 consecutive doubles (B).
constexpr int kStageElems = TM * TK / 256;

struct TileLoad {
    float v[kStageElems];
    __device__ __forceinline__ void load(const float *src, i64 s_row, i64 s_k, int r0, int rows, int k0, int ke) {
#pragma unroll
        for (int q = 0; q < kStageElems; ++q) {
            const int e = threadIdx.x + 256 * q;
            int rr, kk;
            if (s_k == 1) {
                rr = e / TK, kk = e - rr * TK;
            } else {
                kk = e / TM, rr = e - kk * TM;
            }
            const int r = r0 + rr, k = k0 + kk;
            v[q] = (r < rows && k < ke) ? src[(i64)r * s_row + (i64)k * s_k] : 0.0f;
        }
    }
    __device__ __forceinline__ void store(double (*dst)[TM + 1], i64 s_k) const {
#pragma unroll
        for (int q = 0; q < kStageElems; ++q) {
            const int e = threadIdx.x + 256 * q;
            int rr, kk;
            if (s_k == 1) {
                rr = e / TK, kk = e - rr * TK;
            } else {
                kk = e / TM, rr = e - kk * TM;
            }
            dst[kk][rr] = (double)v[q];
        }
    }
};

__global__ void __launch_bounds__(256) sgemm_kernel(Gemm g, int kchunk) {
    __shared__ double sa[TK][TM + 1], sb[TK][TN + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.x * TM, n0 = blockIdx.y * TN;
    const int kb = blockIdx.z * kchunk, ke = min(g.K, kb + kchunk);
    double acc[4][4] = {};
    TileLoad la, lb;
    if (kb < ke) {
        la.load(g.A, g.sam, g.sak, m0, g.M, kb, ke);
        lb.load(g.B, g.sbn, g.sbk, n0, g.N, kb, ke);
    }
    for (int k0 = kb; k0 < ke; k0 += TK) {
        la.store(sa, g.sak);
        lb.store(sb, g.sbk);
        __syncthreads();
        if (k0 + TK < ke) {
            la.load(g.A, g.sam, g.sak, m0, g.M, k0 + TK, ke);
            lb.load(g.B, g.sbn, g.sbk, n0, g.N, k0 + TK, ke);
        }
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sa[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = sb[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            if (m >= g.M || n >= g.N) continue;
            if (gridDim.z == 1) gemm_store(g, m, n, acc[i][j]);
            else g.ws[((i64)blockIdx.z * g.M + m) * g.N + n] = acc[i][j];
        }
}

// Single-row products (M == 1: column sums, the score-vector gradient):
// lane = output column, the CTA's 8 warps interleave the K range of the
// split with 4 independent f64 partial sums each, combined in a fixed order.
__global__ void __launch_bounds__(256) gemv_kernel(Gemm g, int kchunk) {
    __shared__ double red[8][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int n = blockIdx.x * 32 + lane;
    const int kb = blockIdx.y * kchunk, ke = min(g.K, kb + kchunk);
    double p0 = 0.0, p1 = 0.0, p2 = 0.0, p3 = 0.0;
    if (n < g.N) {
        const float *bcol = g.B + (i64)n * g.sbn;
        int k = kb + w;
        for (; k + 24 < ke; k += 32) {
            p0 = fma((double)g.A[(i64)k * g.sak], (double)bcol[(i64)k * g.sbk], p0);
            p1 = fma((double)g.A[(i64)(k + 8) * g.sak], (double)bcol[(i64)(k + 8) * g.sbk], p1);
            p2 = fma((double)g.A[(i64)(k + 16) * g.sak], (double)bcol[(i64)(k + 16) * g.sbk], p2);
            p3 = fma((double)g.A[(i64)(k + 24) * g.sak], (double)bcol[(i64)(k + 24) * g.sbk], p3);
        }
        for (; k < ke; k += 8) p0 = fma((double)g.A[(i64)k * g.sak], (double)bcol[(i64)k * g.sbk], p0);
    }
    red[w][lane] = (p0 + p1) + (p2 + p3);
    __syncthreads();
    if (w == 0 && n < g.N) {
        double t = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) t += red[i][lane];
        if (gridDim.y == 1) gemm_store(g, 0, n, t);
        else g.ws[(i64)blockIdx.y * g.N + n] = t;
    }
}

// Sums the split partials in split order and stores.
__global__ void sgemm_finish_kernel(Gemm g, int splits) {
    GRID_LOOP(e, (i64)g.M * g.N) {
        double acc = 0.0;
        for (int s = 0; s < splits; ++s) acc += g.ws[(i64)s * g.M * g.N + e];
        const int m = (int)(e / g.N), n = (int)(e - (i64)m * g.N);
        gemm_store(g, m, n, acc);
    }
}

// -------------------------------------------------------------- LSTM --
// kLstmS samples per CTA share the recurrent weights (4H x H, f32) in shared
// memory; the recurrent state of every sample is kept there as f64, so each
// f64 multiply-add converts only the weight, once for all kLstmS samples.
// The H-long (forward) or 4H-long (backward) dot products run as independent
// partial sums (even / odd k forward; four lanes per output backward) so the
// f64 chains stay short, and the samples give each thread kLstmS
// independent chains.  Samples never interact inside a recurrence.
constexpr int kLstmS = 4, kLstmRows = 2;

struct LstmFwdPair {
    LstmFwdDir d[2];
};
struct LstmBwdPair {
    LstmBwdDir d[2];
};

__global__ void __launch_bounds__(256) lstm_fwd_kernel(LstmFwdPair dp, int B, int T, int H, float *cat) {
    const LstmFwdDir D = blockIdx.y ? dp.d[1] : dp.d[0];
    const float *xg = D.xg, *b_ih = D.b_ih, *b_hh = D.b_hh, *w_hh = D.w_hh;
    float *gates = D.gates, *c_tr = D.c, *h_prev_tr = D.h_prev;
    const int rev = D.rev, dir = D.dir;
    constexpr int S = kLstmS;
    extern __shared__ double smd[];
    const int G4 = 4 * H;
    double *hb = smd;                                    // [S][H] h of the previous step
    float *wT = reinterpret_cast<float *>(hb + S * H);   // [H][4H]: wT[k*4H + o] = w_hh[o*H + k]
    float *cb = wT + H * G4;                             // [S][H]
    float *gb = cb + S * H;                              // [S][4H]
    const int b0 = blockIdx.x * S;
    const int ns = min(S, B - b0);
    for (int e = threadIdx.x; e < G4 * H; e += blockDim.x) {
        const int o = e / H, k = e - o * H;
        wT[k * G4 + o] = w_hh[e];
    }
    for (int e = threadIdx.x; e < S * H; e += blockDim.x) {
        hb[e] = 0.0;
        cb[e] = 0.0f;
    }
    __syncthreads();
    // The input projections of step st + 1 are read while step st runs (they
    // do not depend on the recurrence), so the global-memory latency stays
    // off the per-step critical path.  Threads own gate rows o = threadIdx.x
    // + k * blockDim.x; kLstmRows bounds k (4H <= kLstmRows * blockDim).
    float xn[kLstmRows][S];
    auto load_xg = [&](int step) {
        const int tq = rev ? T - 1 - step : step;
#pragma unroll
        for (int j = 0; j < kLstmRows; ++j) {
            const int o = threadIdx.x + j * blockDim.x;
#pragma unroll
            for (int q = 0; q < S; ++q)
                xn[j][q] = (o < G4 && q < ns) ? xg[((i64)(b0 + q) * T + tq) * G4 + o] : 0.0f;
        }
    };
    load_xg(0);
    for (int st = 0; st < T; ++st) {
        const int tt = rev ? T - 1 - st : st;
        float xc[kLstmRows][S];
#pragma unroll
        for (int j = 0; j < kLstmRows; ++j)
#pragma unroll
            for (int q = 0; q < S; ++q) xc[j][q] = xn[j][q];
        if (st + 1 < T) load_xg(st + 1);
#pragma unroll
        for (int j = 0; j < kLstmRows; ++j) {
            const int o = threadIdx.x + j * blockDim.x;
            if (o >= G4) break;
            double a0[S], a1[S];
#pragma unroll
            for (int q = 0; q < S; ++q) a0[q] = a1[q] = 0.0;
            int k = 0;
            for (; k + 1 < H; k += 2) {
                const double w0 = (double)wT[k * G4 + o], w1 = (double)wT[(k + 1) * G4 + o];
#pragma unroll
                for (int q = 0; q < S; ++q) {
                    a0[q] = fma(hb[q * H + k], w0, a0[q]);
                    a1[q] = fma(hb[q * H + k + 1], w1, a1[q]);
                }
            }
            if (k < H) {
                const double w0 = (double)wT[k * G4 + o];
#pragma unroll
                for (int q = 0; q < S; ++q) a0[q] = fma(hb[q * H + k], w0, a0[q]);
            }
            const float bias = fadd(b_ih[o], b_hh[o]);
#pragma unroll
            for (int q = 0; q < S; ++q) {
                if (q >= ns) break;
                gb[q * G4 + o] = fadd(fadd(bias, xc[j][q]), (float)(a0[q] + a1[q]));
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < ns * H; e += blockDim.x) {
            const int q = e / H, i = e - q * H;
            const i64 r = (i64)(b0 + q) * T + tt;
            const float *g = gb + q * G4;
            const float ig = sigm(g[i]), fg = sigm(g[H + i]), cg = cr_tanhf(g[2 * H + i]), og = sigm(g[3 * H + i]);
            const float cn = fadd(fmul(fg, cb[e]), fmul(ig, cg));
            const float hn = fmul(og, cr_tanhf(cn));
            gates[r * G4 + i] = ig;
            gates[r * G4 + H + i] = fg;
            gates[r * G4 + 2 * H + i] = cg;
            gates[r * G4 + 3 * H + i] = og;
            c_tr[r * H + i] = cn;
            h_prev_tr[r * H + i] = (float)hb[e];
            cat[r * 2 * H + dir * H + i] = hn;
            cb[e] = cn;
            hb[e] = (double)hn;  // only this thread touches hb[e] in this phase
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(256) lstm_bwd_kernel(LstmBwdPair dp, const float *dcat, int B, int T, int H) {
    const LstmBwdDir D = blockIdx.y ? dp.d[1] : dp.d[0];
    const float *gates = D.gates, *c_tr = D.c, *w_hh = D.w_hh;
    float *dgates = D.dgates;
    const int rev = D.rev, dir = D.dir;
    constexpr int S = kLstmS;
    extern __shared__ double smd[];
    const int G4 = 4 * H;
    double *dgd = smd;                                  // [S][4H] gate gradients of the step, f64
    float *w = reinterpret_cast<float *>(dgd + S * G4);  // [4H][H] natural layout
    float *dhn = w + G4 * H;                            // [S][H]
    float *dcn = dhn + S * H;                           // [S][H]
    const int b0 = blockIdx.x * S;
    const int ns = min(S, B - b0);
    for (int e = threadIdx.x; e < G4 * H; e += blockDim.x) w[e] = w_hh[e];
    for (int e = threadIdx.x; e < S * H; e += blockDim.x) dhn[e] = dcn[e] = 0.0f;
    for (int e = threadIdx.x; e < S * G4; e += blockDim.x) dgd[e] = 0.0;
    __syncthreads();
    // The step's saved gates, cell states and output gradient do not depend
    // on the recurrence: those of step st - 1 are read while step st runs.
    float pf[kLstmRows][7];
    auto load_step = [&](int step) {
        const int tq = rev ? T - 1 - step : step;
        const int tpq = rev ? tq + 1 : tq - 1;
#pragma unroll
        for (int j = 0; j < kLstmRows; ++j) {
            const int e = threadIdx.x + j * blockDim.x;
            if (e >= ns * H) break;
            const int q = e / H, i = e - q * H;
            const i64 r = (i64)(b0 + q) * T + tq;
            pf[j][0] = gates[r * G4 + i];
            pf[j][1] = gates[r * G4 + H + i];
            pf[j][2] = gates[r * G4 + 2 * H + i];
            pf[j][3] = gates[r * G4 + 3 * H + i];
            pf[j][4] = c_tr[r * H + i];
            pf[j][5] = step > 0 ? c_tr[((i64)(b0 + q) * T + tpq) * H + i] : 0.0f;
            pf[j][6] = dcat[r * 2 * H + dir * H + i];
        }
    };
    load_step(T - 1);
    for (int st = T - 1; st >= 0; --st) {
        const int tt = rev ? T - 1 - st : st;
        float cur[kLstmRows][7];
#pragma unroll
        for (int j = 0; j < kLstmRows; ++j)
#pragma unroll
            for (int u = 0; u < 7; ++u) cur[j][u] = pf[j][u];
        if (st > 0) load_step(st - 1);
#pragma unroll
        for (int j = 0; j < kLstmRows; ++j) {
            const int e = threadIdx.x + j * blockDim.x;
            if (e >= ns * H) break;
            const int q = e / H, i = e - q * H;
            const int b = b0 + q;
            const i64 r = (i64)b * T + tt;
            const float ig = cur[j][0], fg = cur[j][1], cg = cur[j][2], og = cur[j][3];
            const float tc = cr_tanhf(cur[j][4]);
            const float cp = cur[j][5];
            const float dh = fadd(cur[j][6], dhn[e]);
            const float dc = fadd(fmul(fmul(dh, og), fsub(1.0f, fmul(tc, tc))), fmul(dcn[e], fg));
            const float d0 = fmul(fmul(fmul(dc, cg), ig), fsub(1.0f, ig));
            const float d1 = fmul(fmul(fmul(dc, cp), fg), fsub(1.0f, fg));
            const float d2 = fmul(fmul(dc, ig), fsub(1.0f, fmul(cg, cg)));
            const float d3 = fmul(fmul(fmul(dh, tc), og), fsub(1.0f, og));
            dgates[r * G4 + i] = d0;
            dgates[r * G4 + H + i] = d1;
            dgates[r * G4 + 2 * H + i] = d2;
            dgates[r * G4 + 3 * H + i] = d3;
            double *dq = dgd + q * G4;
            dq[i] = (double)d0;
            dq[H + i] = (double)d1;
            dq[2 * H + i] = (double)d2;
            dq[3 * H + i] = (double)d3;
            dcn[e] = dc;
        }
        __syncthreads();
        // dh_prev[k] = sum_o dg[o] w[o, k]: four consecutive lanes per k, each
        // over o = q, q + 4, ..., combined with two shuffles
        for (int e = threadIdx.x; e < 4 * H; e += blockDim.x) {
            const int k = e >> 2, l = e & 3;
            double acc[S];
#pragma unroll
            for (int q = 0; q < S; ++q) acc[q] = 0.0;
            for (int o = l; o < G4; o += 4) {
                const double wv = (double)w[o * H + k];
#pragma unroll
                for (int q = 0; q < S; ++q) acc[q] = fma(dgd[q * G4 + o], wv, acc[q]);
            }
#pragma unroll
            for (int q = 0; q < S; ++q) {
                double v = acc[q];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (l == 0 && q < ns) dhn[q * H + k] = (float)v;
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------ attention dec --
// Attention decoder.  A CTA runs kAttnS samples through all decoder steps
// with every thread busy: the recurrent weights sit in shared memory once per
// CTA, each phase of a step spreads its (sample, output) pairs over all
// threads, and the T- or H-long reductions that feed a single value run
// across a warp.  Dot products accumulate in f64 and round once; the
// element-wise expressions keep the reference's f32 order.
constexpr int kAttnS = 4, kAttnThreads = 512;
constexpr size_t kAttnMaxSmem = 227 * 1024;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// sum_k x[k] * w[k * stride] over k < n, f64, two interleaved partial sums.
__device__ __forceinline__ double dot2_d(const float *x, const float *w, int stride, int n) {
    double a0 = 0.0, a1 = 0.0;
    int k = 0;
    for (; k + 1 < n; k += 2) {
        a0 = fma((double)x[k], (double)w[(i64)k * stride], a0);
        a1 = fma((double)x[k + 1], (double)w[(i64)(k + 1) * stride], a1);
    }
    if (k < n) a0 = fma((double)x[k], (double)w[(i64)k * stride], a0);
    return a0 + a1;
}

// Shared-memory layout of the decoder kernels.  The per-step vectors that
// feed dot products (h, context, gate gradients, ...) are kept as f64 copies
// laid out [k][sample], so that a dot product converts only its weight (an
// f32 -> f64 conversion runs on the SM's narrow conversion pipe, which bounds
// these kernels), and a thread that owns one weight column serves every
// sample of the CTA with one conversion per weight.
// DECODE = false: teacher-forced forward of the training step (tokens from
// text_in, every trace stored).  DECODE = true: greedy decoding
// (src/attn.rs:368-447): the token fed at step s is the argmax (first
// maximum) of the generator logits of step s-1, sos at step 0; only the
// per-step argmax tokens are stored.
// stage bit 0: the CTA's encoder projections [S][T][H] are copied into
// shared memory once (read at every step); bit 1: the encoder features too.
constexpr int kAttnRows = 4;  // (sample, t) rows whose warp reductions overlap

__host__ __device__ inline size_t attn_fwd_smem_base(int H, int T, int V, bool decode) {
    const int S = kAttnS, G4 = 4 * H;
    return sizeof(double) * ((size_t)2 * H * S + S * T + H) +
           sizeof(float) * ((size_t)9 * H * H + 16 + 4 * S * H + S * G4 + 2 * S * T + S + (decode ? S * V : 0));
}

template <bool DECODE>
__global__ void __launch_bounds__(kAttnThreads) attn_fwd_kernel(AttnFwd a, int stage) {
    extern __shared__ __align__(16) double attn_smd[];
    const int H = a.H, T = a.T, V = a.V, G4 = 4 * H, CV = H + V;
    constexpr int S = kAttnS;
    double *hd = attn_smd;        // [H][S] h as f64
    double *ctxd = hd + H * S;    // [H][S] context as f64
    double *ald = ctxd + H * S;   // [S][T] alpha as f64
    double *swd = ald + S * T;    // [H] score weights as f64
    float *wihT = reinterpret_cast<float *>(swd + H);  // [H][4H], context columns of w_ih, transposed
    float *whhT = wihT + H * G4 + 16;  // [H][4H] (16 floats apart: the two arrays fall in different banks)
    float *h2hT = whhT + H * G4;       // [H][H]:  h2hT[j*H + k] = h2h_w[k*H + j]
    float *h = h2hT + H * H;           // [S][H]
    float *c = h + S * H, *phh = c + S * H, *ctx = phh + S * H;  // [S][H]
    float *pre = ctx + S * H;     // [S][4H]
    float *e = pre + S * G4;      // [S][T]
    float *al = e + S * T;        // [S][T]
    int *tok = reinterpret_cast<int *>(al + S * T);  // [S]
    float *logit = reinterpret_cast<float *>(tok + S);  // [S][V] (DECODE)
    float *sph = logit + (DECODE ? S * V : 0);
    float *sbh = sph + ((stage & 1) ? S * T * H : 0);
    const int b0 = blockIdx.x * S;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int i = threadIdx.x; i < G4 * H; i += blockDim.x) {
        const int o = i / H, k = i - o * H;
        wihT[k * G4 + o] = a.w_ih[(i64)o * CV + k];
        whhT[k * G4 + o] = a.w_hh[i];
    }
    for (int i = threadIdx.x; i < H * H; i += blockDim.x) {
        const int k = i / H, j = i - k * H;
        h2hT[j * H + k] = a.h2h_w[i];
    }
    for (int i = threadIdx.x; i < S * T * H; i += blockDim.x) {
        const int sl = i / (T * H), r = i - sl * T * H;
        const i64 g = (i64)min(b0 + sl, a.B - 1) * T * H + r;
        if (stage & 1) sph[i] = a.proj_h[g];
        if (stage & 2) sbh[i] = a.bh[g];
    }
    for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
        h[i] = c[i] = 0.0f;
        hd[i] = 0.0;
    }
    for (int k = threadIdx.x; k < H; k += blockDim.x) swd[k] = (double)a.score_w[k];
    if (DECODE && threadIdx.x < S) tok[threadIdx.x] = a.sos;
    __syncthreads();
    for (int st = 0; st < a.steps; ++st) {
        // proj_hh = h2h(h) + bias
        for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
            const int sl = i / H, k = i - sl * H;
            double a0 = 0.0, a1 = 0.0;
            int j = 0;
            for (; j + 1 < H; j += 2) {
                a0 = fma(hd[j * S + sl], (double)h2hT[j * H + k], a0);
                a1 = fma(hd[(j + 1) * S + sl], (double)h2hT[(j + 1) * H + k], a1);
            }
            if (j < H) a0 = fma(hd[j * S + sl], (double)h2hT[j * H + k], a0);
            phh[i] = fadd((float)(a0 + a1), a.h2h_b[k]);
        }
        if (!DECODE && threadIdx.x < S) {
            const int b = min(b0 + (int)threadIdx.x, a.B - 1);
            tok[threadIdx.x] = a.text_in[(i64)b * a.steps + st];
        }
        __syncthreads();
        // tanh(proj_H + proj_hh) and the scores e = tanh(.) . score_w, one
        // warp per (sample, t) row, kAttnRows rows' reductions overlapped
        for (int p0 = warp; p0 < S * T; p0 += nwarps * kAttnRows) {
            double acc[kAttnRows];
#pragma unroll
            for (int u = 0; u < kAttnRows; ++u) {
                acc[u] = 0.0;
                const int p = p0 + u * nwarps;
                if (p < S * T) {
                    const int sl = p / T, t = p - sl * T, b = b0 + sl;
                    const float *php = (stage & 1) ? sph + p * H : a.proj_h + ((i64)min(b, a.B - 1) * T + t) * H;
                    for (int k = lane; k < H; k += 32) {
                        const float v = cr_tanhf(fadd(php[k], phh[sl * H + k]));
                        if (!DECODE && b < a.B) a.tanh_tr[(((i64)st * a.B + b) * T + t) * H + k] = v;
                        acc[u] = fma((double)v, swd[k], acc[u]);
                    }
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < kAttnRows; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < kAttnRows; ++u)
                    if (p0 + u * nwarps < S * T) e[p0 + u * nwarps] = (float)acc[u];
            }
        }
        __syncthreads();
        // softmax over T, one warp per sample
        for (int sl = warp; sl < S; sl += nwarps) {
            float mx = -INFINITY;
            for (int t = lane; t < T; t += 32) mx = fmaxf(mx, e[sl * T + t]);
            mx = warp_max_f(mx);
            double sum = 0.0;
            for (int t = lane; t < T; t += 32) {
                const float v = cr_expf(fsub(e[sl * T + t], mx));
                al[sl * T + t] = v;
                sum += (double)v;
            }
            const float sf = (float)warp_sum_d(sum);
            const int b = b0 + sl;
            for (int t = lane; t < T; t += 32) {
                const float v = fdiv(al[sl * T + t], sf);
                al[sl * T + t] = v;
                ald[sl * T + t] = (double)v;
                if (!DECODE && b < a.B) a.alpha[((i64)st * a.B + b) * T + t] = v;
            }
        }
        __syncthreads();
        // context and the decoder cell input [ctx, one-hot token]
        for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
            const int sl = i / H, k = i - sl * H;
            const int b = min(b0 + sl, a.B - 1);
            const float *bp = (stage & 2) ? sbh + sl * T * H + k : a.bh + (i64)b * T * H + k;
            double acc = 0.0;
            for (int t = 0; t < T; ++t) acc = fma(ald[sl * T + t], (double)bp[t * H], acc);
            const float cv = (float)acc;
            ctx[i] = cv;
            ctxd[k * S + sl] = (double)cv;
        }
        __syncthreads();
        if (!DECODE) {
            for (int i = threadIdx.x; i < S * CV; i += blockDim.x) {
                const int sl = i / CV, j = i - sl * CV, b = b0 + sl;
                if (b < a.B)
                    a.cell_in[((i64)st * a.B + b) * CV + j] =
                        j < H ? ctx[sl * H + j] : (j - H == tok[sl] ? 1.0f : 0.0f);
            }
        }
        // gate pre-activations: (b_ih + b_hh) + w_ih[:, :H] ctx + w_ih[:, H + tok] + w_hh h.
        // Lane pair (2o, 2o+1) owns gate row o: the even lane the context dot,
        // the odd lane the recurrent dot, both for all S samples (two f64
        // partial sums over even and odd k, added at the end); a shuffle
        // swaps the halves and each lane finishes S/2 samples.
        for (int i = threadIdx.x; i < 2 * G4; i += blockDim.x) {
            const int o = i >> 1, dsel = i & 1;
            const float *wcol = (dsel ? whhT : wihT) + o;
            const double *xd = dsel ? hd : ctxd;
            double a0[S], a1[S];
#pragma unroll
            for (int q = 0; q < S; ++q) a0[q] = a1[q] = 0.0;
            int k = 0;
            for (; k + 1 < H; k += 2) {
                const double w0 = (double)wcol[k * G4], w1 = (double)wcol[(k + 1) * G4];
                const double2 *x0 = reinterpret_cast<const double2 *>(xd + k * S);
                const double2 *x1 = reinterpret_cast<const double2 *>(xd + (k + 1) * S);
#pragma unroll
                for (int q = 0; q < S / 2; ++q) {
                    const double2 u0 = x0[q], u1 = x1[q];
                    a0[2 * q] = fma(u0.x, w0, a0[2 * q]);
                    a0[2 * q + 1] = fma(u0.y, w0, a0[2 * q + 1]);
                    a1[2 * q] = fma(u1.x, w1, a1[2 * q]);
                    a1[2 * q + 1] = fma(u1.y, w1, a1[2 * q + 1]);
                }
            }
            if (k < H) {
                const double w0 = (double)wcol[k * G4];
#pragma unroll
                for (int q = 0; q < S; ++q) a0[q] = fma(xd[k * S + q], w0, a0[q]);
            }
            const float bsum = fadd(a.b_ih[o], a.b_hh[o]);
#pragma unroll
            for (int q = 0; q < S; ++q) {
                const double mine = a0[q] + a1[q];
                const double other = __shfl_xor_sync(0xffffffffu, mine, 1);
                if ((q >= S / 2) == (dsel != 0)) {
                    const double dc = dsel ? other : mine, dh = dsel ? mine : other;
                    pre[q * G4 + o] = fadd(fadd(fadd(bsum, (float)dc), a.w_ih[(i64)o * CV + H + tok[q]]), (float)dh);
                }
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
            const int sl = i / H, k = i - sl * H, b = b0 + sl;
            const float *pg = pre + sl * G4;
            const float ig = sigm(pg[k]), fg = sigm(pg[H + k]), cg = cr_tanhf(pg[2 * H + k]), og = sigm(pg[3 * H + k]);
            const float cn = fadd(fmul(fg, c[i]), fmul(ig, cg));
            const float hn = fmul(og, cr_tanhf(cn));
            if (!DECODE && b < a.B) {
                const i64 sb = (i64)st * a.B + b;
                a.gates[sb * G4 + k] = ig;
                a.gates[sb * G4 + H + k] = fg;
                a.gates[sb * G4 + 2 * H + k] = cg;
                a.gates[sb * G4 + 3 * H + k] = og;
                a.cs[sb * H + k] = cn;
                a.hs[sb * H + k] = hn;
            }
            c[i] = cn;
            h[i] = hn;
            hd[k * S + sl] = (double)hn;
        }
        __syncthreads();
        if (DECODE) {
            // generator logits = gen_w h + gen_b (the training path's GEMM
            // expression: f64 dot rounded once, then the bias)
            for (int i = threadIdx.x; i < S * V; i += blockDim.x) {
                const int sl = i / V, v = i - sl * V;
                logit[i] = fadd((float)dot2_d(h + sl * H, a.gen_w + (i64)v * H, 1, H), a.gen_b[v]);
            }
            __syncthreads();
            // argmax, first maximum, one warp per sample
            for (int sl = warp; sl < S; sl += nwarps) {
                float bv = -INFINITY;
                int bi = V;
                for (int v = lane; v < V; v += 32) {
                    const float x = logit[sl * V + v];
                    if (x > bv) {
                        bv = x;
                        bi = v;
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    const int best = bi < V ? bi : 0;  // nothing above -inf: the reference keeps 0
                    tok[sl] = best;
                    if (b0 + sl < a.B) a.step_tokens[(i64)st * a.B + b0 + sl] = best;
                }
            }
            __syncthreads();
        }
    }
}

__host__ __device__ inline size_t attn_bwd_smem_base(int H, int T) {
    const int S = kAttnS, G4 = 4 * H;
    return sizeof(double) * ((size_t)G4 * S + 2 * H * S) +
           sizeof(float) * ((size_t)9 * H * H + 4 * S * H + 3 * S * T + 2 * S * T * H);
}

__global__ void __launch_bounds__(kAttnThreads) attn_bwd_kernel(AttnBwd a, int stage) {
    extern __shared__ __align__(16) double attn_smd[];
    const int H = a.H, T = a.T, V = a.V, G4 = 4 * H, CV = H + V;
    constexpr int S = kAttnS;
    double *dgd = attn_smd;          // [4H][S] gate gradients as f64
    double *dctxd = dgd + G4 * S;    // [H][S] d context as f64
    double *dphhd = dctxd + H * S;   // [H][S] d proj_hh as f64
    float *wc = reinterpret_cast<float *>(dphhd + H * S);  // [4H][H] context columns of w_ih
    float *whh = wc + G4 * H;        // [4H][H]
    float *h2h = whh + G4 * H;       // [H][H]
    float *dhn = h2h + H * H;        // [S][H]
    float *dcn = dhn + S * H, *dctx = dcn + S * H, *dhp = dctx + S * H;  // [S][H]
    float *da = dhp + S * H, *de = da + S * T;                            // [S][T]
    float *acc_bh = de + S * T, *acc_ph = acc_bh + S * T * H;             // [S][T][H]
    float *als = acc_ph + S * T * H;                                      // [S][T] alpha of the step
    float *sbh = als + S * T;                                             // [S][T][H] when stage != 0
    const int b0 = blockIdx.x * S;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int i = threadIdx.x; i < G4 * H; i += blockDim.x) {
        const int o = i / H, k = i - o * H;
        wc[i] = a.w_ih[(i64)o * CV + k];
        whh[i] = a.w_hh[i];
    }
    for (int i = threadIdx.x; i < H * H; i += blockDim.x) h2h[i] = a.h2h_w[i];
    for (int i = threadIdx.x; i < S * H; i += blockDim.x) dhn[i] = dcn[i] = 0.0f;
    for (int i = threadIdx.x; i < S * T * H; i += blockDim.x) {
        acc_bh[i] = acc_ph[i] = 0.0f;
        if (stage) {
            const int sl = i / (T * H), r = i - sl * T * H;
            sbh[i] = a.bh[(i64)min(b0 + sl, a.B - 1) * T * H + r];
        }
    }
    __syncthreads();
    for (int st = a.steps - 1; st >= 0; --st) {
        for (int i = threadIdx.x; i < S * T; i += blockDim.x) {
            const int sl = i / T, t = i - sl * T;
            als[i] = a.alpha[((i64)st * a.B + min(b0 + sl, a.B - 1)) * T + t];
        }
        // LSTM cell backward
        for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
            const int sl = i / H, k = i - sl * H, b = min(b0 + sl, a.B - 1);
            const i64 sb = (i64)st * a.B + b;
            const float *g = a.gates + sb * G4;
            const float ig = g[k], fg = g[H + k], cg = g[2 * H + k], og = g[3 * H + k];
            const float tc = cr_tanhf(a.cs[sb * H + k]);
            const float cp = st > 0 ? a.cs[(sb - a.B) * H + k] : 0.0f;
            const float dh = fadd(a.d_out_hid[sb * H + k], dhn[i]);
            const float dc = fadd(fmul(fmul(dh, og), fsub(1.0f, fmul(tc, tc))), fmul(dcn[i], fg));
            dgd[k * S + sl] = (double)fmul(fmul(fmul(dc, cg), ig), fsub(1.0f, ig));
            dgd[(H + k) * S + sl] = (double)fmul(fmul(fmul(dc, cp), fg), fsub(1.0f, fg));
            dgd[(2 * H + k) * S + sl] = (double)fmul(fmul(dc, ig), fsub(1.0f, fmul(cg, cg)));
            dgd[(3 * H + k) * S + sl] = (double)fmul(fmul(fmul(dh, tc), og), fsub(1.0f, og));
            dcn[i] = dc;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < S * G4; i += blockDim.x) {
            const int sl = i / G4, o = i - sl * G4, b = b0 + sl;
            if (b < a.B) a.dgates[((i64)st * a.B + b) * G4 + o] = (float)dgd[o * S + sl];
        }
        // d ctx = w_ih[:, :H]^T dg, d h_prev (direct) = w_hh^T dg.  Item
        // ((dot, half, k), parity): the f64 partial sum over the gate rows o
        // of one parity for the samples of one half; the lane pair adds its
        // even and odd partial sums.
        for (int i = threadIdx.x; i < 8 * H; i += blockDim.x) {
            const int parity = i & 1, r = i >> 1;
            const int k = r % H, dh2 = r / H, half = dh2 & 1, dsel = dh2 >> 1;
            const float *wm = (dsel ? whh : wc) + k;
            double s0 = 0.0, s1 = 0.0;
            for (int o = parity; o < G4; o += 2) {
                const double w = (double)wm[o * H];
                const double2 x = *reinterpret_cast<const double2 *>(dgd + o * S + 2 * half);
                s0 = fma(x.x, w, s0);
                s1 = fma(x.y, w, s1);
            }
            const double t0 = s0 + __shfl_xor_sync(0xffffffffu, s0, 1);
            const double t1 = s1 + __shfl_xor_sync(0xffffffffu, s1, 1);
            if (parity == 0) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int sl = 2 * half + q;
                    const float v = (float)(q ? t1 : t0);
                    if (dsel) {
                        dhp[sl * H + k] = v;
                    } else {
                        dctx[sl * H + k] = v;
                        dctxd[k * S + sl] = (double)v;
                    }
                }
            }
        }
        __syncthreads();
        // d alpha = d ctx . bh[t] and acc_bh += alpha * d ctx, one warp per
        // (sample, t) row, kAttnRows rows' reductions overlapped
        for (int p0 = warp; p0 < S * T; p0 += nwarps * kAttnRows) {
            double acc[kAttnRows];
#pragma unroll
            for (int u = 0; u < kAttnRows; ++u) {
                acc[u] = 0.0;
                const int p = p0 + u * nwarps;
                if (p < S * T) {
                    const int sl = p / T, t = p - sl * T, b = min(b0 + sl, a.B - 1);
                    const float *bht = stage ? sbh + p * H : a.bh + ((i64)b * T + t) * H;
                    const float alv = als[p];
                    for (int k = lane; k < H; k += 32) {
                        acc[u] = fma(dctxd[k * S + sl], (double)bht[k], acc[u]);
                        acc_bh[p * H + k] = fadd(acc_bh[p * H + k], fmul(alv, dctx[sl * H + k]));
                    }
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < kAttnRows; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < kAttnRows; ++u)
                    if (p0 + u * nwarps < S * T) da[p0 + u * nwarps] = (float)acc[u];
            }
        }
        __syncthreads();
        // softmax backward, one warp per sample: de = alpha (d alpha - alpha . d alpha)
        for (int sl = warp; sl < S; sl += nwarps) {
            const int b = min(b0 + sl, a.B - 1);
            const float *al = als + sl * T;
            double acc = 0.0;
            for (int t = lane; t < T; t += 32) acc = fma((double)al[t], (double)da[sl * T + t], acc);
            const float dt = (float)warp_sum_d(acc);
            for (int t = lane; t < T; t += 32) {
                const float v = fmul(al[t], fsub(da[sl * T + t], dt));
                de[sl * T + t] = v;
                if (b0 + sl < a.B) a.de[((i64)st * a.B + b) * T + t] = v;
            }
        }
        __syncthreads();
        // through tanh, one (sample, k) per thread over t: acc_ph += de *
        // score_w * (1 - tn^2) (a zero de leaves acc_ph as it is), d proj_hh
        // = the f64 sum of the same terms over t
        for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
            const int sl = i / H, k = i - sl * H, b = min(b0 + sl, a.B - 1);
            const float *tn = a.tanh_tr + (((i64)st * a.B + b) * T) * H;
            const float sw = a.score_w[k];
            double sum = 0.0;
            for (int t = 0; t < T; ++t) {
                const float v = tn[t * H + k];
                const float d = de[sl * T + t];
                const float term = fmul(fmul(d, sw), fsub(1.0f, fmul(v, v)));
                if (d != 0.0f) acc_ph[(sl * T + t) * H + k] = fadd(acc_ph[(sl * T + t) * H + k], term);
                sum += (double)term;
            }
            dphhd[k * S + sl] = (double)(float)sum;
            if (b0 + sl < a.B) a.dprojhh[((i64)st * a.B + b) * H + k] = (float)sum;
        }
        __syncthreads();
        // d h_prev += h2h^T d proj_hh
        for (int i = threadIdx.x; i < S * H; i += blockDim.x) {
            const int sl = i / H, j = i - sl * H;
            double a0 = 0.0, a1 = 0.0;
            int k = 0;
            for (; k + 1 < H; k += 2) {
                a0 = fma(dphhd[k * S + sl], (double)h2h[k * H + j], a0);
                a1 = fma(dphhd[(k + 1) * S + sl], (double)h2h[(k + 1) * H + j], a1);
            }
            if (k < H) a0 = fma(dphhd[k * S + sl], (double)h2h[k * H + j], a0);
            dhn[i] = fadd(dhp[i], (float)(a0 + a1));
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < S * T * H; i += blockDim.x) {
        const int sl = i / (T * H), r = i - sl * T * H, b = b0 + sl;
        if (b >= a.B) continue;
        a.d_proj_h[(i64)b * T * H + r] = acc_ph[i];
        a.d_bh[(i64)b * T * H + r] = acc_bh[i];
    }
}

// ------------------------------------------------------------ losses --
__global__ void ce_rows_kernel(const float *logits, const int32_t *target, int B, int steps, int V, int pad,
                               float *d, float *row_loss) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= B * steps) return;
    const int st = warp / B, b = warp - st * B;
    const float *x = logits + (i64)warp * V;
    float *dr = d + (i64)warp * V;
    const int tgt = target[(i64)b * steps + st];
    if (tgt == pad) {
        for (int k = lane; k < V; k += 32) dr[k] = 0.0f;
        if (lane == 0) row_loss[warp] = 0.0f;
        return;
    }
    float mx = -INFINITY;
    for (int k = lane; k < V; k += 32) mx = fmaxf(mx, x[k]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double sd = 0.0;
    for (int k = lane; k < V; k += 32) sd += (double)cr_expf(fsub(x[k], mx));
    for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
    const float s = (float)sd;
    for (int k = lane; k < V; k += 32) {
        const float p = fdiv(cr_expf(fsub(x[k], mx)), s);
        dr[k] = k == tgt ? fsub(p, 1.0f) : p;
    }
    if (lane == 0) row_loss[warp] = -cr_logf(fdiv(cr_expf(fsub(x[tgt], mx)), s));
}

__device__ __forceinline__ double logadd(double a, double b) {
    if (a == -INFINITY) return b;
    if (b == -INFINITY) return a;
    return a > b ? a + log(1.0 + exp(b - a)) : b + log(1.0 + exp(a - b));
}

__device__ bool ctc_valid(const int32_t *len, int b, int T) { return len[b] > 0 && T >= len[b] + 1; }

__global__ void ctc_kernel(const float *logits, const int32_t *tgt, const int32_t *len, int Lmax, int B, int T, int V,
                           float cw, float *grad, double *sample_loss) {
    extern __shared__ double smd[];
    const int b = blockIdx.x;
    const int L = len[b];
    const int S = 2 * L + 1;
    double *al = smd, *be = al + (i64)T * (2 * Lmax + 1);
    float *lp = reinterpret_cast<float *>(be + (i64)T * (2 * Lmax + 1));  // [T][V]
    int *ext = reinterpret_cast<int *>(lp + T * V);
    __shared__ double loss_s;
    __shared__ int n_valid;
    float *g = grad + (i64)b * T * V;
    if (!ctc_valid(len, b, T)) {  // zero_infinity: no loss, zero gradient
        for (int i = threadIdx.x; i < T * V; i += blockDim.x) g[i] = 0.0f;
        if (threadIdx.x == 0) sample_loss[b] = 0.0;
        return;
    }
    if (threadIdx.x == 0) {
        int n = 0;
        for (int i = 0; i < B; ++i) n += ctc_valid(len, i, T) ? 1 : 0;
        n_valid = n > 0 ? n : 1;
    }
    for (int s = threadIdx.x; s < S; s += blockDim.x) ext[s] = (s & 1) ? tgt[(i64)b * Lmax + (s >> 1)] : 0;
    // log-softmax rows (src/ctc.rs:1-19): f32 max, f64 sum of exp, f32 result
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float *x = logits + ((i64)b * T + t) * V;
        float mx = -INFINITY;
        for (int k = 0; k < V; ++k) mx = fmaxf(mx, x[k]);
        double se = 0.0;
        for (int k = 0; k < V; ++k) se += exp((double)fsub(x[k], mx));
        const double ls = log(se);
        for (int k = 0; k < V; ++k) lp[t * V + k] = (float)((double)x[k] - (double)mx - ls);
    }
    __syncthreads();
    const int SS = 2 * Lmax + 1;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
        al[s] = s < 2 ? (double)lp[ext[s]] : -INFINITY;
        be[(T - 1) * SS + s] = s >= S - 2 ? 0.0 : -INFINITY;
    }
    __syncthreads();
    for (int t = 1; t < T; ++t) {  // src/ctc.rs:49-73
        for (int s = threadIdx.x; s < S; s += blockDim.x) {
            double best = al[(t - 1) * SS + s];
            if (s > 0) best = logadd(best, al[(t - 1) * SS + s - 1]);
            if (s >= 2 && ext[s - 2] != ext[s]) best = logadd(best, al[(t - 1) * SS + s - 2]);
            al[t * SS + s] = best + (double)lp[t * V + ext[s]];
        }
        __syncthreads();
    }
    for (int t = T - 2; t >= 0; --t) {  // src/ctc.rs:75-100
        for (int s = threadIdx.x; s < S; s += blockDim.x) {
            const float *row = lp + (t + 1) * V;
            double best = be[(t + 1) * SS + s] + (double)row[ext[s]];
            if (s + 1 < S) best = logadd(best, be[(t + 1) * SS + s + 1] + (double)row[ext[s + 1]]);
            if (s + 2 < S && ext[s + 2] != ext[s]) best = logadd(best, be[(t + 1) * SS + s + 2] + (double)row[ext[s + 2]]);
            be[t * SS + s] = best;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) loss_s = -logadd(al[(T - 1) * SS + S - 1], al[(T - 1) * SS + S - 2]);
    __syncthreads();
    const double loss = loss_s;
    if (!isfinite(loss)) {
        for (int i = threadIdx.x; i < T * V; i += blockDim.x) g[i] = 0.0f;
        if (threadIdx.x == 0) sample_loss[b] = 0.0;
        return;
    }
    const double scale = 1.0 / ((double)L * (double)n_valid);
    for (int i = threadIdx.x; i < T * V; i += blockDim.x) {
        const int t = i / V, k = i - t * V;
        double gam = 0.0;
        for (int s = 0; s < S; ++s)
            if (ext[s] == k) gam += exp(al[t * SS + s] + be[t * SS + s] + loss);
        const double p = (double)cr_expf(lp[i]);
        g[i] = fmul((float)((p - gam) * scale), cw);
    }
    if (threadIdx.x == 0) sample_loss[b] = loss / (double)L;
}

__global__ void loss_finalize_kernel(const float *row_loss, const int32_t *target, int B, int steps, int pad,
                                     const double *sample_loss, const int32_t *ctc_len, int T, float cw, float *out,
                                     float *scale_out) {
    __shared__ double sa[32], sc[32];
    __shared__ int cnt[32], nv[32];
    double a = 0.0, c = 0.0;
    int k = 0, n = 0;
    for (int i = threadIdx.x; i < B * steps; i += blockDim.x) {
        const int st = i / B, b = i - st * B;
        if (target[(i64)b * steps + st] != pad) {
            ++k;
            a += (double)row_loss[i];
        }
    }
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        c += sample_loss[b];
        n += ctc_valid(ctc_len, b, T) ? 1 : 0;
    }
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        c += __shfl_xor_sync(0xffffffffu, c, o);
        k += __shfl_xor_sync(0xffffffffu, k, o);
        n += __shfl_xor_sync(0xffffffffu, n, o);
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sa[w] = a; sc[w] = c; cnt[w] = k; nv[w] = n; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double A = 0.0, Cc = 0.0;
        int K = 0, N = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { A += sa[i]; Cc += sc[i]; K += cnt[i]; N += nv[i]; }
        K = K > 0 ? K : 1;
        N = N > 0 ? N : 1;
        const double attn = A / K, ctc = Cc / N;
        out[0] = (float)((double)fsub(1.0f, cw) * attn + (double)cw * ctc);
        out[1] = (float)attn;
        out[2] = (float)ctc;
        *scale_out = fdiv(fsub(1.0f, cw), (float)K);
    }
}

__global__ void scale_by_kernel(float *x, const float *s, i64 n) {
    const float v = *s;
    GRID_LOOP(i, n) x[i] = fmul(x[i], v);
}

}  // namespace

void sgemm(const Gemm &g, cudaStream_t st) {
    if (g.M <= 0 || g.N <= 0) return;
    if (g.M == 1) {
        const int nb = (g.N + 31) / 32;
        int splits = 1;
        if (g.ws && g.K > 256) {
            const int want = (4 * sm_count() + nb - 1) / nb;
            const int maxs = (g.K + 255) / 256;
            splits = want < maxs ? want : maxs;
            if ((i64)splits * g.N > g.ws_elems) splits = (int)(g.ws_elems / g.N);
            if (splits < 1) splits = 1;
        }
        const int kchunk = (g.K + splits - 1) / splits;
        splits = (g.K + kchunk - 1) / kchunk;
        if (splits < 1) splits = 1;
        gemv_kernel<<<dim3(nb, splits), 256, 0, st>>>(g, kchunk > 0 ? kchunk : 1);
        TRBA_LAUNCH_CHECK();
        if (splits > 1) {
            sgemm_finish_kernel<<<grid_for((i64)g.N), 256, 0, st>>>(g, splits);
            TRBA_LAUNCH_CHECK();
        }
        return;
    }
    const int mt = (g.M + TM - 1) / TM, nt = (g.N + TN - 1) / TN;
    // Split K until the grid covers four CTAs per SM (chunks of >= 64).
    int splits = 1;
    if (g.ws && g.K > 128) {
        const int want = (4 * sm_count() + mt * nt - 1) / (mt * nt);
        const int maxs = (g.K + 63) / 64;
        splits = want < maxs ? want : maxs;
        if ((i64)splits * g.M * g.N > g.ws_elems) splits = (int)(g.ws_elems / ((i64)g.M * g.N));
        if (splits < 1) splits = 1;
    }
    int kchunk = (g.K + splits - 1) / splits;
    kchunk = (kchunk + TK - 1) / TK * TK;
    splits = (g.K + kchunk - 1) / kchunk;
    if (splits < 1) splits = 1;
    sgemm_kernel<<<dim3(mt, nt, splits), 256, 0, st>>>(g, kchunk > 0 ? kchunk : TK);
    TRBA_LAUNCH_CHECK();
    if (splits > 1) {
        sgemm_finish_kernel<<<grid_for((i64)g.M * g.N), 256, 0, st>>>(g, splits);
        TRBA_LAUNCH_CHECK();
    }
}

void col_sums(const float *X, int rows, int cols, i64 ld, const float *ones, float *out, bool accumulate, double *ws,
              i64 ws_elems, cudaStream_t st) {
    Gemm g;
    g.M = 1, g.N = cols, g.K = rows;
    g.A = ones, g.sam = 0, g.sak = 1;
    g.B = X, g.sbk = ld, g.sbn = 1;
    g.C = out, g.ldc = cols;
    g.accumulate = accumulate;
    g.ws = ws, g.ws_elems = ws_elems;
    sgemm(g, st);
}

static void set_smem(const void *fn, size_t bytes) {
    if (bytes > 48 * 1024) TRBA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

void lstm_fwd(const LstmFwdDir *dirs, int ndir, int B, int T, int H, float *cat, cudaStream_t st) {
    TRBA_REQUIRE(ndir == 1 || ndir == 2, "lstm_fwd: one or two directions per launch");
    const size_t smem = sizeof(double) * kLstmS * H + sizeof(float) * ((size_t)4 * H * H + kLstmS * H + kLstmS * 4 * H);
    TRBA_REQUIRE(smem <= 200 * 1024, "lstm_fwd: hidden size too large for the shared-memory recurrence");
    TRBA_REQUIRE(4 * H <= kLstmRows * 256, "lstm_fwd: at most 2 gate rows per thread (hidden <= 128)");
    set_smem((const void *)lstm_fwd_kernel, smem);
    LstmFwdPair dp{};
    dp.d[0] = dirs[0];
    dp.d[1] = dirs[ndir - 1];
    lstm_fwd_kernel<<<dim3((B + kLstmS - 1) / kLstmS, ndir), 256, smem, st>>>(dp, B, T, H, cat);
    TRBA_LAUNCH_CHECK();
}

void lstm_bwd(const LstmBwdDir *dirs, int ndir, const float *dcat, int B, int T, int H, cudaStream_t st) {
    TRBA_REQUIRE(ndir == 1 || ndir == 2, "lstm_bwd: one or two directions per launch");
    TRBA_REQUIRE(H % 8 == 0, "lstm_bwd: hidden size must be a multiple of 8 (4*hidden fills whole warps)");
    const size_t smem = sizeof(double) * kLstmS * 4 * H + sizeof(float) * ((size_t)4 * H * H + 2 * kLstmS * H);
    TRBA_REQUIRE(smem <= 200 * 1024, "lstm_bwd: hidden size too large for the shared-memory recurrence");
    TRBA_REQUIRE(kLstmS * H <= kLstmRows * 256, "lstm_bwd: at most 2 state rows per thread (hidden <= 128)");
    set_smem((const void *)lstm_bwd_kernel, smem);
    LstmBwdPair dp{};
    dp.d[0] = dirs[0];
    dp.d[1] = dirs[ndir - 1];
    lstm_bwd_kernel<<<dim3((B + kLstmS - 1) / kLstmS, ndir), 256, smem, st>>>(dp, dcat, B, T, H);
    TRBA_LAUNCH_CHECK();
}

static int attn_fwd_stage(size_t base, size_t block, size_t *total) {
    int stage = 0;
    *total = base;
    if (*total + block <= kAttnMaxSmem) stage |= 1, *total += block;
    if (*total + block <= kAttnMaxSmem) stage |= 2, *total += block;
    return stage;
}

void attn_fwd(const AttnFwd &a, cudaStream_t st) {
    const int H = a.H, T = a.T, S = kAttnS;
    TRBA_REQUIRE(H % 4 == 0, "attn_fwd: hidden size must be a multiple of 4 (gate rows fill whole warps)");
    size_t total = 0;
    const int stage = attn_fwd_stage(attn_fwd_smem_base(H, T, a.V, false), sizeof(float) * (size_t)S * T * H, &total);
    TRBA_REQUIRE(total <= kAttnMaxSmem, "attn_fwd: hidden / encoder length too large for shared memory");
    set_smem((const void *)attn_fwd_kernel<false>, total);
    attn_fwd_kernel<false><<<(a.B + S - 1) / S, kAttnThreads, total, st>>>(a, stage);
    TRBA_LAUNCH_CHECK();
}

void attn_decode(const AttnFwd &a, cudaStream_t st) {
    const int H = a.H, T = a.T, S = kAttnS;
    TRBA_REQUIRE(H % 4 == 0, "attn_decode: hidden size must be a multiple of 4 (gate rows fill whole warps)");
    size_t total = 0;
    const int stage = attn_fwd_stage(attn_fwd_smem_base(H, T, a.V, true), sizeof(float) * (size_t)S * T * H, &total);
    TRBA_REQUIRE(total <= kAttnMaxSmem, "attn_decode: hidden / encoder length too large for shared memory");
    set_smem((const void *)attn_fwd_kernel<true>, total);
    attn_fwd_kernel<true><<<(a.B + S - 1) / S, kAttnThreads, total, st>>>(a, stage);
    TRBA_LAUNCH_CHECK();
}

void attn_bwd(const AttnBwd &a, cudaStream_t st) {
    const int H = a.H, T = a.T, S = kAttnS;
    TRBA_REQUIRE(H % 4 == 0, "attn_bwd: hidden size must be a multiple of 4 (gate-gradient items fill whole warps)");
    const size_t smem = attn_bwd_smem_base(H, T);
    const size_t stage_bytes = sizeof(float) * (size_t)S * T * H;
    const int stage = smem + stage_bytes <= kAttnMaxSmem ? 1 : 0;
    const size_t total = smem + (stage ? stage_bytes : 0);
    TRBA_REQUIRE(total <= kAttnMaxSmem, "attn_bwd: hidden / encoder length too large for shared memory");
    set_smem((const void *)attn_bwd_kernel, total);
    attn_bwd_kernel<<<(a.B + S - 1) / S, kAttnThreads, total, st>>>(a, stage);
    TRBA_LAUNCH_CHECK();
}

void ce_rows(const float *logits, const int32_t *target, int B, int steps, int V, int pad, float *d_logits,
             float *row_loss, cudaStream_t st) {
    const int rows = B * steps;
    ce_rows_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(logits, target, B, steps, V, pad, d_logits, row_loss);
    TRBA_LAUNCH_CHECK();
}

void ctc(const float *logits, const int32_t *ctc_tgt, const int32_t *ctc_len, int Lmax, int B, int T, int V, float cw,
         float *grad, double *sample_loss, cudaStream_t st) {
    const size_t smem = sizeof(double) * 2 * (size_t)T * (2 * Lmax + 1) + sizeof(float) * (size_t)T * V +
                        sizeof(int) * (2 * Lmax + 1);
    set_smem((const void *)ctc_kernel, smem);
    ctc_kernel<<<B, 128, smem, st>>>(logits, ctc_tgt, ctc_len, Lmax, B, T, V, cw, grad, sample_loss);
    TRBA_LAUNCH_CHECK();
}

void loss_finalize(const float *row_loss, const int32_t *target, int B, int steps, int pad, const double *sample_loss,
                   const int32_t *ctc_len, int T, float cw, float *d_logits, int V, float *out, cudaStream_t st) {
    loss_finalize_kernel<<<1, 1024, 0, st>>>(row_loss, target, B, steps, pad, sample_loss, ctc_len, T, cw, out,
                                             out + 3);
    TRBA_LAUNCH_CHECK();
    const i64 n = (i64)B * steps * V;
    scale_by_kernel<<<grid_for(n), 256, 0, st>>>(d_logits, out + 3, n);
    TRBA_LAUNCH_CHECK();
}

}  // namespace seq
}  // namespace trba

// ---------------------------------------------------------------------------
// GEMM entry point that allocates nothing.
//
// Some callers cannot call cudaMalloc: plugins whose host framework owns every
// device allocation, or latency-critical loops in which cudaMalloc / cudaFree
// would synchronise the device.  trba_sgemm_exact_noalloc gives them the
// f64-accumulated, split-K fp32 GEMM of the training step without any
// allocation: the split-K partial sums live in the file-scope array below.
//
// Limits and behaviour:
//   * the scratch array holds kNoAllocScratch doubles (8 MiB); every GPU that
//     loads this library keeps it for the life of the process;
//   * at most kNoAllocMaxOut = M*N outputs per call; larger calls are
//     rejected with an error (nothing is launched);
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) — make that first call
//     before any stream capture;
//   * every call shares the one array and finds the previous call's partial
//     sums in it; each call overwrites every element it later reads, so no
//     clearing is needed, but calls that overlap on the GPU (different
//     streams, different host threads) race on the array and must be
//     serialised by the caller.
// ---------------------------------------------------------------------------
namespace {

constexpr long long kNoAllocScratch = 1LL << 20;  // doubles
constexpr long long kNoAllocMaxOut = 1LL << 17;   // M * N

__device__ __align__(256) double g_noalloc_scratch[kNoAllocScratch];

// Device address of the scratch array, looked up once per device.  Host
// threads may call the entry point concurrently, so the cache entries are
// atomics (a racing first lookup stores the same address twice).  A cached
// address stays valid for the life of the device's primary context; after a
// cudaDeviceReset the library must be reloaded.
std::atomic<double *> g_noalloc_ptr[64];

}  // namespace

extern "C" int trba_sgemm_exact_noalloc(const float *a, const float *b, float *c, int m, int n, int k, void *stream) {
    using namespace trba;
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    if ((long long)m * n > kNoAllocMaxOut) {
        report_error(__FILE__, __LINE__,
                     "trba_sgemm_exact_noalloc: M*N exceeds the 131072 outputs its static scratch supports", -1);
        return -1;
    }
    int dev = 0;
    const cudaError_t de = cudaGetDevice(&dev);
    if (de != cudaSuccess || dev < 0 || dev >= 64) {
        report_error(__FILE__, __LINE__, "trba_sgemm_exact_noalloc: no current device", (int)de);
        return de != cudaSuccess ? (int)de : -1;
    }
    double *ws = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (!ws) {  // once per device, with that device current
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            report_error(__FILE__, __LINE__, "trba_sgemm_exact_noalloc: cudaGetSymbolAddress failed", (int)e);
            return e != cudaSuccess ? (int)e : -1;
        }
        ws = static_cast<double *>(p);
        g_noalloc_ptr[dev].store(ws, std::memory_order_relaxed);
    }
    seq::Gemm g;
    g.M = m, g.N = n, g.K = k;
    g.A = a, g.sam = k, g.sak = 1;  // A [M, K] row-major
    g.B = b, g.sbk = n, g.sbn = 1;  // B [K, N] row-major
    g.C = c, g.ldc = n;             // C [M, N] compact
    g.ws = ws;
    g.ws_elems = kNoAllocScratch;
    seq::sgemm(g, as_stream(stream));
    const cudaError_t le = cudaGetLastError();
    return le == cudaSuccess ? 0 : (int)le;
}
