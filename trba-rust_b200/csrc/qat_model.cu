// Device-resident TRBA INT8-QAT training step (include/trba_qat.h).
//
// Model: SE-ResNet QAT backbone (src/qnet.rs:1425-1758), BiLSTM stack
// (src/rnn.rs), attention decoder (src/attn.rs), CTC head (LinearF), losses
// and optimiser of return_main_step (later snapshot src/main.rs:2249-2413).
// Every buffer is allocated once at creation for the largest batch; a step
// launches kernels only (no allocation, no host synchronisation), so the
// whole step can be enqueued back to back and, in data-parallel mode, the
// gradient buffer is all-reduced with one NCCL call.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>
#include <string>
#include <vector>

#include "common.cuh"
#include "conv_implicit.cuh"
#include "dgrad_tc.cuh"
#include "gemm_i8.cuh"
#include "qat_kernels.cuh"
#include "seq_kernels.cuh"
#include "trba_backend.h"
#include "trba_qat.h"

using namespace trba;

namespace {

// NCCL is resolved at run time (dlopen) rather than linked: a process that
// already holds a libnccl.so.2 (PyTorch bundles one) keeps using that copy,
// and a process that never goes data-parallel never loads NCCL at all.
struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    bool ok = false;
};

const Nccl &nccl() {
    static Nccl n;
    static bool tried = false;
    if (tried) return n;
    tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return n;
    n.GetUniqueId = (decltype(n.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    n.CommInitRank = (decltype(n.CommInitRank))dlsym(h, "ncclCommInitRank");
    n.AllReduce = (decltype(n.AllReduce))dlsym(h, "ncclAllReduce");
    n.CommDestroy = (decltype(n.CommDestroy))dlsym(h, "ncclCommDestroy");
    n.GetErrorString = (decltype(n.GetErrorString))dlsym(h, "ncclGetErrorString");
    n.CommGetAsyncError = (decltype(n.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
    n.CommAbort = (decltype(n.CommAbort))dlsym(h, "ncclCommAbort");
    n.ok = n.GetUniqueId && n.CommInitRank && n.AllReduce && n.CommDestroy && n.GetErrorString &&
           n.CommGetAsyncError && n.CommAbort;
    return n;
}

__host__ __device__ inline int a16(int x) { return (x + 15) & ~15; }
inline i64 a16l(i64 x) { return (x + 15) & ~15LL; }

// ----------------------------------------------------------- allocation --
struct Arena {
    char *base = nullptr;
    size_t cap = 0, used = 0;
    std::vector<std::pair<size_t, size_t>> plan;  // (offset, bytes) while planning
    bool planning = true;
    size_t take(size_t bytes) {
        size_t off = (used + 255) & ~size_t(255);
        used = off + bytes;
        return off;
    }
};

template <typename T>
struct Ref {  // arena-relative pointer, resolved after the single cudaMalloc (null: never allocated)
    size_t off = 0;
    Arena *a = nullptr;
    T *get() const { return a ? reinterpret_cast<T *>(a->base + off) : nullptr; }
};

enum Kind { K_CONV = 0, K_MAT = 1, K_VEC = 2 };

struct Entry {
    std::string name;
    i64 off;
    int rows, cols, kind;
    i64 size() const { return cols ? (i64)rows * cols : rows; }
};

struct Seg {  // a parameter segment for the multi-tensor optimiser kernels
    i64 off;
    int n;
    int rows, cols;
    int aux;  // conv: index into conv tables
    int chan; // conv: offset of its first output channel among all convs' channels
};

struct ConvL {
    std::string name;
    int cin, cout, kh, kw, sh, sw, ph, pw;
    int H, W, Ho, Wo;
    int K, kp;
    i64 w_off, gamma_off, beta_off;
    // persistent
    Ref<int8_t> wq;          // [a16(cout), kp]
    // Implicit-GEMM forward (Cin a power of two >= 16): the operand is gathered
    // from the NHWC copy of the input; wqh = the weights in (ky, kx, ci) K order
    bool implicit = false;
    Ref<int8_t> wqh;         // [cout, K]
    Ref<float> wT;           // (float) wq in the input-gradient layout (dgrad_weights_index), exact mode
    dgtc::Plan tc;           // tensor-core input gradient: class plan (tc_ok) and its bf16 weight image
    bool tc_ok = false;
    Ref<uint8_t> wimg;
    Ref<dgtc::Plan> d_tc;
    std::vector<int> cls_perm, cls_start;  // tap-class pixel order of the input gradient (empty: natural)
    Ref<int32_t> d_perm, d_cstart;
    Ref<float> ws, wmax;     // device scalars
    Ref<float> run_mean, run_var;
    // forward traces
    Ref<int8_t> col, colT;   // [a16(rows), kp] / [a16(K), a16(rows)]; implicit convs: training only
    Ref<float> x, mean, var, y;
    Ref<int8_t> q;           // quantised output (when the conv is followed by relu_quant)
    Ref<float> s_q;          // its scale
    const int8_t *q_in = nullptr;  // resolved per step
    const float *s_in = nullptr;
    // per-step zeroed
    Ref<double> bn_acc, bwd_acc;
    Ref<float> ymax, dxmax, s_dx;
    Ref<int32_t> gw;
    // backward
    Ref<int8_t> A;           // [a16(cout), a16(rows)]
    bool need_y = false, need_q = false;
    i64 rows(int B) const { return (i64)B * Ho * Wo; }
};

struct BlockL {
    int c1, c2, ds;  // conv indices (ds = -1 if none)
    int C, Cin, H, W, Ho, Wo, R;
    i64 w1_off, w2_off;
    Ref<float> pool, h1, gate, s_out, zmax, gvmax, s_dq;
    Ref<int8_t> q_out;
    Ref<float> dz, dy2, dy1, gin, dpre1, dpre2, dpooled;
};

struct RnnL {
    int D, H;
    i64 wih[2], bih[2], whh[2], bhh[2], pw, pb;
    Ref<float> xg[2], gates[2], c[2], hprev[2], dg[2];
    Ref<float> cat, y, dcat, dx;
};

// Kernel probe: CUDA events around every launch of one kernel family, on
// the stream the step runs on, so that a timed loop can report that family's
// device time per launch live (trba_model_probe / trba_model_probe_read).
constexpr size_t kProbeStamps = 256;

__global__ void stamp_kernel(unsigned long long *dst) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    *dst = t;
}

struct Probe {
    int kind = -1;
    std::vector<cudaEvent_t> ev;  // start/stop pairs
    size_t used = 0;
    double ops = 0.0;    // algorithmic arithmetic operations of the timed launches
    double bytes = 0.0;  // algorithmic bytes (one read of every input, one write of every output)
    long long launches = 0;
    long long steps = 0;  // steps recorded while probing (a step graph records one)
    // Inside a step graph the launches are bracketed by device timestamps
    // (%globaltimer, written by a one-thread kernel on the same stream)
    // instead of events: a graph-recorded event cannot be timed.
    unsigned long long *stamps = nullptr;  // [2 * kProbeStamps] device
    size_t nstamp = 0;
    bool stamped = false;
};

}  // namespace

struct trba_model {
    trba_model_config cfg;
    int B = 0;  // max batch
    int T = 0, steps = 0, Hf = 0;
    std::vector<Entry> manifest;
    i64 n_params = 0;
    std::vector<ConvL> convs;
    std::vector<BlockL> blocks;
    std::vector<RnnL> rnn;
    Arena arena, zarena;  // persistent / zeroed every step
    // parameters, gradients, Adam moments
    Ref<float> P, G, Mm, Vv;
    // stem
    Ref<int8_t> qpool;
    Ref<int8_t> qh;          // NHWC copy of the current implicit conv's input
    Ref<float> s_img;
    Ref<float> dy_c1, dy_c0, gv_last, dy_o1, dy_o0;
    // features and sequence head
    Ref<float> feat, dfeat;
    Ref<float> proj_h, tanh_tr, alpha, cell_in, agates, hs, cs, logits, dlogits, row_loss, ctc_logits, dctc;
    Ref<float> d_out_hid, adg, ade, adprojhh, d_proj_h, d_bh;
    Ref<double> ctc_sample_loss;
    Ref<double> gemm_ws;   // split-K partial sums of the fp32 GEMMs
    Ref<uint16_t> dg_planes;  // tensor-core input gradient: dy as three bf16 planes (largest conv's dy)
    i64 gemm_ws_elems = 0;
    Ref<float> ones;       // column-sum helper
    Ref<float> loss;  // 4 floats
    Ref<int32_t> step_tokens;  // [steps, B]: greedy-decoding argmax of every step (inference)
    // optimiser scratch (zeroed per step)
    Ref<double> gsq_total;
    Ref<double> conv_gsq;  // per conv
    Ref<unsigned> wmax_bits;  // per conv (per output channel in per-channel mode): max |w| as f32 bits,
                              // cleared before each re-quantisation
    int n_chan = 0;           // output channels of all convs
    Ref<float> clip_f, mat_step, conv_step;
    Ref<double> step_state;  // [t, clip active, bc1, bc2]: advanced on the device every step
    // inputs staged for the host-buffer entry point
    Ref<int8_t> in_img;
    Ref<int32_t> in_text, in_target, in_ctc, in_ctc_len;
    // segment tables
    std::vector<Seg> vec_segs, mat_segs, conv_segs;
    Seg *d_vec = nullptr, *d_mat = nullptr, *d_conv = nullptr;
    // conv tables for multi-conv kernels
    struct ConvTab {
        int8_t *wq;
        float *ws, *wmax;
        float *mean, *var, *run_mean, *run_var;
        int cout, K, kp;
        float *wT;  // null in tensor-core mode
        int khw;
        const dgtc::Plan *tc;  // tensor-core mode: the plan (device copy) and the image it writes
        uint8_t *wimg;
        int per_channel;       // per-output-channel weight scales (ws, wmax hold cout values)
        int8_t *wqh;           // implicit-GEMM forward: [cout, K] in (ky, kx, ci) order, or null
    };
    ConvTab *d_convtab = nullptr;
    long long t = 0;
    int last_B = 0;
    ncclComm_t comm = nullptr;
    int world = 1;
    cudaEvent_t ev = nullptr;
    // Weight-gradient stream of the conv backward: every conv's BN backward
    // chain and weight-gradient GEMM run there (forked when the conv's dy is
    // ready, joined once after the last conv), while the chain of input
    // gradients runs on the step's stream.
    cudaStream_t side = nullptr;
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    // CUDA-graph execution of the whole step (trba_model_use_graphs): the
    // graph is recorded on gstream for one set of input pointers and batch.
    bool use_graphs = false;
    cudaStream_t gstream = nullptr;
    cudaEvent_t gfork = nullptr, gjoin = nullptr;
    cudaGraphExec_t gexec = nullptr;
    const void *gkey[5] = {};
    int gkey_batch = 0, gkey_probe = -1;
    long long graph_kernels = 0;  // kernel launches recorded in the step graph
    Probe probe;
};

namespace {

// ------------------------------------------------- optimiser kernels --
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void sumsq_kernel(const float *g, i64 n, double *out) {
    __shared__ double sm[32];
    double s = 0.0;
    GRID_LOOP(i, n) s += (double)g[i] * (double)g[i];
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0;
        s = warp_sum_d(s);
        if (threadIdx.x == 0) atomicAdd(out, s);
    }
}

// src/main.rs:2382-2390: f = 5 / (norm + 1e-6) when norm > 5, else 1.
// Rust f32::powi (LLVM __powisf2): square-and-multiply in f32.
__device__ float powi_dev(float a, long long n) {
    float r = 1.0f;
    while (true) {
        if (n & 1) r = fmul(r, a);
        n >>= 1;
        if (n == 0) return r;
        a = fmul(a, a);
    }
}

// Advances the optimiser's step state on the device: clip is active while the
// step count before this step is below clip_warmup; the Adam bias corrections
// (src/opt.rs) use the count after it.  st = [t, clip active, bc1, bc2].
__global__ void step_state_kernel(double *st, int clip_warmup) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        const long long t0 = (long long)st[0];
        st[1] = t0 < clip_warmup ? 1.0 : 0.0;
        const long long t = t0 + 1;
        st[0] = (double)t;
        st[2] = 1.0 - (double)powi_dev(0.9f, t);
        st[3] = 1.0 - (double)powi_dev(0.999f, t);
    }
}

__global__ void clip_factor_kernel(const double *gsq, const double *st, float *f) {
    if (threadIdx.x == 0) {
        float v = 1.0f;
        if (st[1] != 0.0) {
            const double norm = sqrt(*gsq);
            if (norm > 5.0) v = (float)(5.0 / (norm + 1e-6));
        }
        *f = v;
    }
}

// Adam on vector parameters (src/opt.rs adam_vec with the grads scaled by f:
// the same arithmetic as launch_adam_f32 with clip = f).
__global__ void adam_segs_kernel(const Seg *segs, float *P, const float *G, float *M, float *V, const float *f,
                                 double lr, double wd, double b1, double b2, double eps, const double *st) {
    const Seg s = segs[blockIdx.y];
    const double clip = (double)*f;
    const double bc1 = st[2], bc2 = st[3];
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < s.n; j += gridDim.x * blockDim.x) {
        const i64 i = s.off + j;
        const double gi = __dadd_rn((double)(float)__dmul_rn((double)G[i], clip), __dmul_rn(wd, (double)P[i]));
        const float mf = (float)__dadd_rn(__dmul_rn(b1, (double)M[i]), __dmul_rn(1.0 - b1, gi));
        const float vf = (float)__dadd_rn(__dmul_rn(b2, (double)V[i]), __dmul_rn(__dmul_rn(1.0 - b2, gi), gi));
        M[i] = mf;
        V[i] = vf;
        const double mh = __ddiv_rn((double)mf, bc1), vh = __ddiv_rn((double)vf, bc2);
        P[i] = fsub(P[i], (float)__ddiv_rn(__dmul_rn(lr, mh), __dadd_rn(__dsqrt_rn(vh), eps)));
    }
}

// Host Muon (src/opt.rs muon_step_f32) on grads scaled by f: one CTA per
// matrix computes ||g||^2 in f32 and the step lr*sqrt(max)*min(sqrt(min)/frob, cap).
__global__ void muon_mat_norm_kernel(const Seg *segs, const float *G, const float *f, float lr, float cap,
                                     float *step) {
    __shared__ double sm[32];
    const Seg s = segs[blockIdx.x];
    const float fv = *f;
    double acc = 0.0;  // ||f g||^2 accumulated in f64, rounded once
    for (int j = threadIdx.x; j < s.n; j += blockDim.x) {
        const float g = fmul(G[s.off + j], fv);
        acc += (double)fmul(g, g);
    }
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double td = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) td += sm[w];
        const float t = (float)td;
        const float frob = fmaxf(__fsqrt_rn(t), 1e-8f);
        const float mn = (float)min(s.rows, s.cols), mx = (float)max(s.rows, s.cols);
        const float scale = fminf(fdiv(__fsqrt_rn(mn), frob), cap);
        step[blockIdx.x] = fmul(fmul(lr, __fsqrt_rn(mx)), scale);
    }
}

__global__ void muon_mat_apply_kernel(const Seg *segs, float *P, const float *G, const float *f, const float *step,
                                      float dec) {
    const Seg s = segs[blockIdx.y];
    const float fv = *f, st = step[blockIdx.y];
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < s.n; j += gridDim.x * blockDim.x) {
        const i64 i = s.off + j;
        const float u = fsub(fmul(P[i], dec), fmul(st, fmul(G[i], fv)));
        P[i] = isfinite(u) ? u : 0.0f;
    }
}

// Device conv Muon (later snapshot cpu_backend.cpp:1197-1213 /
// src/qnet.rs:559-573): per conv gsq = sum g^2 (f64, unscaled grads), step =
// (float)(clip * lr sqrt(max) * min(sqrt(min)/||g||, cap)).
__global__ void conv_gsq_kernel(const Seg *segs, const float *G, double *gsq) {
    __shared__ double sm[32];
    const Seg s = segs[blockIdx.y];
    double acc = 0.0;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < s.n; j += gridDim.x * blockDim.x) {
        const double v = (double)G[s.off + j];
        acc += v * v;
    }
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        acc = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.0;
        acc = warp_sum_d(acc);
        if (threadIdx.x == 0) atomicAdd(gsq + blockIdx.y, acc);
    }
}

__global__ void conv_muon_apply_kernel(const Seg *segs, float *P, const float *G, const double *gsq, const float *f,
                                       double lr, double wd, double cap) {
    const Seg s = segs[blockIdx.y];
    const double frob = __dsqrt_rn(fmax(gsq[blockIdx.y], 1e-30));
    const double mn = (double)min(s.rows, s.cols), mx = (double)max(s.rows, s.cols);
    const double scale = fmin(__ddiv_rn(__dsqrt_rn(mn), fmax(frob, 1e-8)), cap);
    const double lre = __dmul_rn(lr, __dsqrt_rn(mx));
    const float step = (float)__dmul_rn(__dmul_rn((double)*f, lre), scale);
    const float dec = (float)(1.0 - __dmul_rn(lr, wd));
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < s.n; j += gridDim.x * blockDim.x) {
        const i64 i = s.off + j;
        const float u = fsub(fmul(P[i], dec), fmul(step, G[i]));
        P[i] = isfinite(u) ? u : 0.0f;
    }
}

// Re-quantisation of every conv (src/qnet.rs:601-624): max|w| per conv, then
// the padded int8 operand with s = max/127 (f64; 1 if 0).  The maximum is
// reduced by gridDim.x blocks per conv: each block's max (fmaxf, so NaN is
// ignored as in a sequential fmaxf scan) is merged with an integer atomicMax
// on the f32 bits, which orders non-negative floats exactly.
__global__ void conv_wmax_kernel(const Seg *segs, const float *P, unsigned *wmax_bits) {
    __shared__ float sm[32];
    const Seg s = segs[blockIdx.y];
    float m = 0.0f;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < s.n; j += gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(P[s.off + j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, sm[w]);
        atomicMax(wmax_bits + s.chan, __float_as_uint(t));
    }
}

// Per-output-channel max |w| (per-channel weight quantisation): one warp per
// weight row, rows of every conv in one launch (blockIdx.y = conv).
__global__ void conv_wmax_rows_kernel(const Seg *segs, const float *P, unsigned *wmax_bits) {
    const Seg s = segs[blockIdx.y];
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < s.rows; r += gridDim.x * warps) {
        const float *row = P + s.off + (i64)r * s.cols;
        float m = 0.0f;
        for (int j = lane; j < s.cols; j += 32) m = fmaxf(m, fabsf(row[j]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax_bits[s.chan + r] = __float_as_uint(m);
    }
}

__device__ __forceinline__ int8_t quant_w(float w, float sc) {
    const float v = (float)__ddiv_rn((double)w, (double)sc);
    return (int8_t)roundf(fminf(fmaxf(v, -127.0f), 127.0f));
}

__device__ __forceinline__ float wscale_of(unsigned bits) {
    const double mx = (double)__uint_as_float(bits);
    return (float)(mx > 0.0 ? __ddiv_rn(mx, 127.0) : 1.0);
}

// Writes the padded int8 GEMM operand, the weight scale(s) and the input
// gradient's weights: per tensor, the same int8 values as f32 in the
// [Cin / 16][tap][Cout][16] layout (exact gather) or as the bf16 image of
// the tensor-core kernel.  Per output channel (t.per_channel): row r has
// scale max |w[r]| / 127; the exact gather's f32 weights are then the
// dequantised values wq * w_s[r] (its final scale is 1) and the tensor-core
// image keeps the int8 values (its producer scales dy per channel).
__global__ void conv_quant_kernel(const Seg *segs, const float *P, const trba_model::ConvTab *tab,
                                  const unsigned *wmax_bits) {
    const Seg s = segs[blockIdx.y];
    const trba_model::ConvTab t = tab[s.aux];
    const bool pc = t.per_channel;
    const unsigned *wb = wmax_bits + s.chan;
    if (blockIdx.x == 0) {
        for (int r = threadIdx.x; r < (pc ? t.cout : 1); r += blockDim.x) {
            t.wmax[r] = __uint_as_float(wb[r]);
            t.ws[r] = wscale_of(wb[r]);
        }
    }
    const float sc0 = wscale_of(wb[0]);
    const i64 total = (i64)a16(t.cout) * t.kp;
    for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (i64)gridDim.x * blockDim.x) {
        const int r = (int)(e / t.kp), c = (int)(e - (i64)r * t.kp);
        t.wq[e] = (r < t.cout && c < t.K) ? quant_w(P[s.off + (i64)r * t.K + c], pc ? wscale_of(wb[r]) : sc0)
                                          : (int8_t)0;
    }
    if (t.wqh) {  // implicit-GEMM forward: K order (ky, kx, ci)
        const int cin = t.K / t.khw;
        const i64 nh = (i64)t.cout * t.K;
        for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < nh; e += (i64)gridDim.x * blockDim.x) {
            const int r = (int)(e / t.K), k = (int)(e - (i64)r * t.K);
            const int tap = k / cin, ci = k - tap * cin;
            t.wqh[e] = quant_w(P[s.off + (i64)r * t.K + (i64)ci * t.khw + tap], pc ? wscale_of(wb[r]) : sc0);
        }
    }
    if (t.wimg) {  // tensor-core input gradient: the bf16 weight image
        const dgtc::Plan &tp = *t.tc;
        const i64 n_img = dgtc::image_elements(tp);
        for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < n_img; e += (i64)gridDim.x * blockDim.x) {
            int co;
            i64 dst;
            const int src = dgtc::image_element(tp, e, co, dst);
            const float v =
                src >= 0 ? (float)quant_w(P[s.off + (i64)co * t.K + src], pc ? wscale_of(wb[co]) : sc0) : 0.0f;
            *reinterpret_cast<__nv_bfloat16 *>(t.wimg + dst) = __float2bfloat16_rn(v);
        }
    }
    if (!t.wT) return;
    const int cin = t.K / t.khw;
    const i64 nT = (i64)((cin + 15) >> 4) * t.khw * t.cout * 16;
    for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < nT; e += (i64)gridDim.x * blockDim.x) {
        const int j = (int)(e & 15);
        const i64 r = e >> 4;
        const int oc = (int)(r % t.cout);
        const i64 r2 = r / t.cout;
        const int tap = (int)(r2 % t.khw), ci = (int)(r2 / t.khw) * 16 + j;
        float v = 0.0f;
        if (ci < cin) {
            const float sc = pc ? wscale_of(wb[oc]) : sc0;
            v = (float)quant_w(P[s.off + (i64)oc * t.K + (i64)ci * t.khw + tap], sc);
            if (pc) v = fmul(v, sc);
        }
        t.wT[e] = v;
    }
}

// BatchNorm running statistics (src/qnet.rs:63-68): r = 0.9 r + 0.1 batch.
__global__ void bn_running_kernel(const trba_model::ConvTab *tab, int nconv) {
    const trba_model::ConvTab t = tab[blockIdx.x];
    for (int c = threadIdx.x; c < t.cout; c += blockDim.x) {
        t.run_mean[c] = fadd(fmul(0.9f, t.run_mean[c]), fmul(0.1f, t.mean[c]));
        t.run_var[c] = fadd(fmul(0.9f, t.run_var[c]), fmul(0.1f, t.var[c]));
    }
    (void)nconv;
}

__global__ void fill_f32_kernel(float *p, i64 n, float v) { GRID_LOOP(i, n) p[i] = v; }

// ----------------------------------------------------------- building --
struct Builder {
    trba_model *m;
    Arena *A, *Z;
    template <typename T>
    Ref<T> take(Arena *ar, i64 count) {
        Ref<T> r;
        r.a = ar;
        r.off = ar->take((size_t)count * sizeof(T));
        return r;
    }
    template <typename T>
    Ref<T> p(i64 n) { return take<T>(A, n); }
    template <typename T>
    Ref<T> z(i64 n) { return take<T>(Z, n); }
    // training-only buffers (gradients, optimiser state, backward traces):
    // not allocated for an inference-only model
    template <typename T>
    Ref<T> tp(i64 n) { return m->cfg.inference_only ? Ref<T>{} : take<T>(A, n); }
    template <typename T>
    Ref<T> tz(i64 n) { return m->cfg.inference_only ? Ref<T>{} : take<T>(Z, n); }
};

void add_entry(trba_model *m, const std::string &name, int rows, int cols, int kind) {
    Entry e{name, m->n_params, rows, cols, kind};
    m->n_params += e.size();
    m->manifest.push_back(e);
}

i64 entry_off(const trba_model *m, const std::string &name) {
    for (auto &e : m->manifest)
        if (e.name == name) return e.off;
    return -1;
}

void plan(trba_model *m) {
    const auto &c = m->cfg;
    const int fd = c.fd;
    const int w[6] = {fd / 8, fd / 4, fd / 2, fd / 2, fd, fd};
    struct BS {
        std::string name;
        int ic, oc, s, li, bi;
    };
    std::vector<BS> bs = {{"layer1.0", w[1], w[2], 2, 0, 0}, {"layer2.0", w[2], w[3], 1, 1, 0},
                          {"layer2.1", w[3], w[3], 1, 1, 1}, {"layer3.0", w[3], w[4], 2, 2, 0}};
    for (int i = 1; i < 5; ++i) bs.push_back({"layer3." + std::to_string(i), w[4], w[4], 1, 2, i});
    for (int i = 0; i < 3; ++i) bs.push_back({"layer4." + std::to_string(i), w[5], w[5], 1, 3, i});

    auto add_conv = [&](const std::string &name, int cin, int cout, int k1, int k2, int s1, int s2, int p1, int p2,
                        int H, int W) -> int {
        ConvL L;
        L.name = name;
        L.cin = cin, L.cout = cout, L.kh = k1, L.kw = k2, L.sh = s1, L.sw = s2, L.ph = p1, L.pw = p2;
        L.H = H, L.W = W;
        L.Ho = (H + 2 * p1 - k1) / s1 + 1;
        L.Wo = (W + 2 * p2 - k2) / s2 + 1;
        L.K = cin * k1 * k2;
        L.kp = a16(L.K);
        // Input-gradient pixel order: grouped by valid taps (strided convs) or
        // by valid kernel rows (stride 1).
        qat::dgrad_classes(H, W, k1, k2, s1, s2, p1, p2, L.Ho, L.Wo, s1 == 1 && s2 == 1, L.cls_perm, L.cls_start);
        L.tc_ok = m->cfg.dgrad_mode == 1 &&
                  dgtc::make_plan(cin, cout, H, W, k1, k2, s1, s2, p1, p2, L.Ho, L.Wo, L.tc);
        L.implicit = m->cfg.conv_fwd_mode == 1 && cin >= 16 && cin <= 1024 && (cin & (cin - 1)) == 0;
        m->convs.push_back(L);
        return (int)m->convs.size() - 1;
    };
    int H = c.img_h, W = c.img_w;
    add_conv("stem.0", 3, w[0], 3, 3, 1, 1, 1, 1, H, W);
    add_conv("stem.3", w[0], w[1], 3, 3, 1, 1, 1, 1, H, W);
    H /= 2;
    W /= 2;
    for (auto &b : bs) {
        BlockL bl;
        bl.ds = -1;
        if (b.s != 1 || b.ic != b.oc) bl.ds = add_conv(b.name + ".downsample.0", b.ic, b.oc, 1, 1, b.s, b.s, 0, 0, H, W);
        bl.c1 = add_conv(b.name + ".conv1", b.ic, b.oc, 3, 3, b.s, b.s, 1, 1, H, W);
        const ConvL &c1 = m->convs[bl.c1];
        bl.c2 = add_conv(b.name + ".conv2", b.oc, b.oc, 3, 3, 1, 1, 1, 1, c1.Ho, c1.Wo);
        bl.C = b.oc, bl.Cin = b.ic, bl.H = H, bl.W = W, bl.Ho = c1.Ho, bl.Wo = c1.Wo, bl.R = b.oc / 16;
        m->blocks.push_back(bl);
        H = bl.Ho;
        W = bl.Wo;
    }
    add_conv("conv_out.0", w[5], w[5], 2, 2, 2, 1, 0, 1, H, W);
    const ConvL &o0 = m->convs.back();
    add_conv("conv_out.3", w[5], w[5], 2, 2, 1, 1, 0, 0, o0.Ho, o0.Wo);
    m->Hf = m->convs.back().Ho;
    m->T = m->convs.back().Wo;
    m->steps = c.max_len + 1;

    // manifest (src/main.rs:954-1030 order)
    for (auto &L : m->convs) {
        add_entry(m, L.name + ".w", L.cout, L.K, K_CONV);
        add_entry(m, L.name + ".gamma", L.cout, 0, K_VEC);
        add_entry(m, L.name + ".beta", L.cout, 0, K_VEC);
    }
    for (size_t i = 0; i < bs.size(); ++i) {
        const std::string pre = "l" + std::to_string(bs[i].li) + "b" + std::to_string(bs[i].bi) + ".se.";
        add_entry(m, pre + "fc1.w", bs[i].oc / 16, bs[i].oc, K_MAT);
        add_entry(m, pre + "fc2.w", bs[i].oc, bs[i].oc / 16, K_MAT);
    }
    const int Hh = c.hidden, V = c.classes;
    for (int li = 0; li < c.rnn_layers; ++li) {
        const int D = li == 0 ? fd : Hh;
        const std::string pre = "rnn" + std::to_string(li) + ".";
        for (const char *dn : {"f", "b"}) {
            add_entry(m, pre + dn + ".w_ih", 4 * Hh, D, K_MAT);
            add_entry(m, pre + dn + ".b_ih", 4 * Hh, 0, K_VEC);
            add_entry(m, pre + dn + ".w_hh", 4 * Hh, Hh, K_MAT);
            add_entry(m, pre + dn + ".b_hh", 4 * Hh, 0, K_VEC);
        }
        add_entry(m, pre + "proj.w", Hh, 2 * Hh, K_MAT);
        add_entry(m, pre + "proj.b", Hh, 0, K_VEC);
    }
    add_entry(m, "attn.i2h.w", Hh, Hh, K_MAT);
    add_entry(m, "attn.h2h.w", Hh, Hh, K_MAT);
    add_entry(m, "attn.h2h.b", Hh, 0, K_VEC);
    add_entry(m, "attn.score.w", 1, Hh, K_MAT);
    add_entry(m, "attn.w_ih", 4 * Hh, Hh + V, K_MAT);
    add_entry(m, "attn.b_ih", 4 * Hh, 0, K_VEC);
    add_entry(m, "attn.w_hh", 4 * Hh, Hh, K_MAT);
    add_entry(m, "attn.b_hh", 4 * Hh, 0, K_VEC);
    add_entry(m, "attn.gen.w", V, Hh, K_MAT);
    add_entry(m, "attn.gen.b", V, 0, K_VEC);
    add_entry(m, "ctc.w", V, Hh, K_MAT);
    add_entry(m, "ctc.b", V, 0, K_VEC);

    for (auto &L : m->convs) {
        L.w_off = entry_off(m, L.name + ".w");
        L.gamma_off = entry_off(m, L.name + ".gamma");
        L.beta_off = entry_off(m, L.name + ".beta");
    }
    for (size_t i = 0; i < bs.size(); ++i) {
        const std::string pre = "l" + std::to_string(bs[i].li) + "b" + std::to_string(bs[i].bi) + ".se.";
        m->blocks[i].w1_off = entry_off(m, pre + "fc1.w");
        m->blocks[i].w2_off = entry_off(m, pre + "fc2.w");
    }
    for (int li = 0; li < c.rnn_layers; ++li) {
        RnnL r;
        r.D = li == 0 ? fd : Hh;
        r.H = Hh;
        const std::string pre = "rnn" + std::to_string(li) + ".";
        const char *dn[2] = {"f", "b"};
        for (int d = 0; d < 2; ++d) {
            r.wih[d] = entry_off(m, pre + dn[d] + ".w_ih");
            r.bih[d] = entry_off(m, pre + dn[d] + ".b_ih");
            r.whh[d] = entry_off(m, pre + dn[d] + ".w_hh");
            r.bhh[d] = entry_off(m, pre + dn[d] + ".b_hh");
        }
        r.pw = entry_off(m, pre + "proj.w");
        r.pb = entry_off(m, pre + "proj.b");
        m->rnn.push_back(r);
    }
    for (auto &e : m->manifest) {
        Seg s{e.off, (int)e.size(), e.rows, e.cols, 0, 0};
        if (e.kind == K_VEC) m->vec_segs.push_back(s);
        else if (e.kind == K_MAT) m->mat_segs.push_back(s);
    }
    for (size_t i = 0; i < m->convs.size(); ++i) {
        const ConvL &L = m->convs[i];
        m->conv_segs.push_back(Seg{L.w_off, L.cout * L.K, L.cout, L.K, (int)i, m->n_chan});
        m->n_chan += L.cout;
    }
}

void allocate(trba_model *m) {
    const auto &c = m->cfg;
    const int B = m->B;
    Builder b{m, &m->arena, &m->zarena};
    m->P = b.p<float>(m->n_params);
    m->G = b.tp<float>(m->n_params);
    m->Mm = b.tp<float>(m->n_params);
    m->Vv = b.tp<float>(m->n_params);
    m->s_img = b.p<float>(1);
    const bool correct = c.wgrad_mode == 1;
    i64 qh_bytes = 0;
    for (size_t i = 0; i < m->convs.size(); ++i) {
        ConvL &L = m->convs[i];
        const i64 rows = L.rows(B), rp = a16l(rows), n = (i64)B * L.cout * L.Ho * L.Wo;
        L.wq = b.p<int8_t>((i64)a16(L.cout) * L.kp);
        if (L.tc_ok) {
            L.wimg = b.tp<uint8_t>(dgtc::weight_image_bytes(L.tc));
            L.d_tc = b.tp<dgtc::Plan>(1);
        } else {
            L.wT = b.tp<float>(qat::dgrad_weights_size(L.cin, L.cout, L.kh * L.kw));
        }
        if (!L.tc_ok && !L.cls_perm.empty()) {
            L.d_perm = b.tp<int32_t>((i64)L.cls_perm.size());
            L.d_cstart = b.tp<int32_t>((i64)L.cls_start.size());
        }
        L.ws = b.p<float>(L.cout);  // per-tensor mode uses ws[0]
        L.wmax = b.p<float>(L.cout);
        L.run_mean = b.p<float>(L.cout);
        L.run_var = b.p<float>(L.cout);
        if (L.implicit) {
            L.wqh = b.p<int8_t>((i64)L.cout * L.K);
            // the im2col matrix: the reference-compatible weight gradient's
            // operand (training only)
            if (!correct) L.col = b.tp<int8_t>(rp * L.kp);
            qh_bytes = std::max(qh_bytes, (i64)B * L.cin * L.H * L.W);
        } else {
            L.col = b.p<int8_t>(rp * L.kp);
        }
        if (correct) L.colT = b.tp<int8_t>((i64)a16(L.K) * rp);
        L.x = b.p<float>(n);
        L.mean = b.p<float>(L.cout);
        L.var = b.p<float>(L.cout);
        L.A = b.tp<int8_t>((i64)a16(L.cout) * rp);
        L.bn_acc = b.z<double>(2 * L.cout);
        L.bwd_acc = b.tz<double>(2 * L.cout);
        L.ymax = b.z<float>(1);
        L.dxmax = b.tz<float>(1);
        L.s_dx = b.tz<float>(1);
        L.gw = b.tz<int32_t>((i64)L.cout * L.K);
    }
    // which convs store y / produce a quantised output
    for (auto &bl : m->blocks) {
        m->convs[bl.c2].need_y = true;
        if (bl.ds >= 0) m->convs[bl.ds].need_y = true;
        m->convs[bl.c1].need_q = true;
    }
    const int nc = (int)m->convs.size();
    for (int i : {0, 1, nc - 2, nc - 1}) m->convs[i].need_q = true;
    for (auto &L : m->convs) {
        const i64 n = (i64)B * L.cout * L.Ho * L.Wo;
        if (L.need_y) L.y = b.p<float>(n);
        if (L.need_q) {
            L.q = b.p<int8_t>(n);
            L.s_q = b.p<float>(1);
        }
    }
    const ConvL &s1 = m->convs[1];
    m->qpool = b.p<int8_t>((i64)B * s1.cout * (s1.Ho / 2) * (s1.Wo / 2));
    if (qh_bytes) m->qh = b.p<int8_t>(qh_bytes);
    for (auto &bl : m->blocks) {
        const i64 n = (i64)B * bl.C * bl.Ho * bl.Wo, nin = (i64)B * bl.Cin * bl.H * bl.W;
        bl.pool = b.p<float>((i64)B * bl.C);
        bl.h1 = b.p<float>((i64)B * bl.R);
        bl.gate = b.p<float>((i64)B * bl.C);
        bl.s_out = b.p<float>(1);
        bl.s_dq = b.p<float>(1);
        bl.q_out = b.p<int8_t>(n);
        bl.zmax = b.z<float>(1);
        bl.gvmax = b.tz<float>(1);
        bl.dz = b.tp<float>(n);
        bl.dy2 = b.tp<float>(n);
        bl.dy1 = b.tp<float>(n);
        bl.gin = b.tp<float>(nin);
        bl.dpre1 = b.tp<float>((i64)B * bl.R);
        bl.dpre2 = b.tp<float>((i64)B * bl.C);
        bl.dpooled = b.tp<float>((i64)B * bl.C);
    }
    const ConvL &o0 = m->convs[nc - 2], &o1 = m->convs[nc - 1];
    m->dy_o1 = b.tp<float>((i64)B * o1.cout * o1.Ho * o1.Wo);
    m->dy_o0 = b.tp<float>((i64)B * o0.cout * o0.Ho * o0.Wo);
    m->gv_last = b.tp<float>((i64)B * o0.cin * o0.H * o0.W);
    m->dy_c1 = b.tp<float>((i64)B * s1.cout * s1.Ho * s1.Wo);
    m->dy_c0 = b.tp<float>((i64)B * m->convs[0].cout * m->convs[0].Ho * m->convs[0].Wo);
    const int T = m->T, Hh = c.hidden, V = c.classes, S = m->steps, fd = c.fd;
    m->feat = b.p<float>((i64)B * T * fd);
    m->dfeat = b.tp<float>((i64)B * T * fd);
    for (auto &r : m->rnn) {
        for (int d = 0; d < 2; ++d) {
            r.xg[d] = b.p<float>((i64)B * T * 4 * Hh);
            r.gates[d] = b.p<float>((i64)B * T * 4 * Hh);
            r.c[d] = b.p<float>((i64)B * T * Hh);
            r.hprev[d] = b.p<float>((i64)B * T * Hh);
            r.dg[d] = b.tp<float>((i64)B * T * 4 * Hh);
        }
        r.cat = b.p<float>((i64)B * T * 2 * Hh);
        r.dcat = b.tp<float>((i64)B * T * 2 * Hh);
        r.y = b.p<float>((i64)B * T * Hh);
        r.dx = b.tp<float>((i64)B * T * r.D);
    }
    m->proj_h = b.p<float>((i64)B * T * Hh);
    m->tanh_tr = b.p<float>((i64)S * B * T * Hh);
    m->alpha = b.p<float>((i64)S * B * T);
    m->cell_in = b.p<float>((i64)S * B * (Hh + V));
    m->agates = b.p<float>((i64)S * B * 4 * Hh);
    m->hs = b.p<float>((i64)S * B * Hh);
    m->cs = b.p<float>((i64)S * B * Hh);
    m->logits = b.p<float>((i64)S * B * V);
    m->dlogits = b.tp<float>((i64)S * B * V);
    m->row_loss = b.p<float>((i64)S * B);
    m->ctc_logits = b.p<float>((i64)B * T * V);
    m->dctc = b.tp<float>((i64)B * T * V);
    m->d_out_hid = b.tp<float>((i64)S * B * Hh);
    m->adg = b.tp<float>((i64)S * B * 4 * Hh);
    m->ade = b.tp<float>((i64)S * B * T);
    m->adprojhh = b.tp<float>((i64)S * B * Hh);
    m->d_proj_h = b.tp<float>((i64)B * T * Hh);
    m->d_bh = b.tp<float>((i64)B * T * Hh);
    m->ctc_sample_loss = b.p<double>(B);
    {
        i64 planes = 0;  // scratch of the tensor-core input gradients, reused conv after conv (one stream)
        for (auto &L : m->convs)
            if (L.tc_ok) {
                dgtc::Plan p = L.tc;
                dgtc::set_batch(p, B);
                planes = std::max(planes, 3 * (i64)dgtc::plane_elements(p));
            }
        if (planes) m->dg_planes = b.tp<uint16_t>(planes);
    }
    m->gemm_ws_elems = (i64)8 << 20;
    m->gemm_ws = b.p<double>(m->gemm_ws_elems);
    m->ones = b.p<float>((i64)B * (S > T ? S : T) * 1);
    m->loss = b.p<float>(4);
    m->step_tokens = b.p<int32_t>((i64)S * B);
    m->gsq_total = b.z<double>(1);
    m->conv_gsq = b.z<double>((i64)m->convs.size());
    m->wmax_bits = b.p<unsigned>((i64)m->n_chan);
    m->clip_f = b.p<float>(1);
    m->step_state = b.p<double>(4);
    m->mat_step = b.p<float>((i64)m->mat_segs.size());
    m->conv_step = b.p<float>((i64)m->convs.size());
    m->in_img = b.p<int8_t>((i64)B * 3 * c.img_h * c.img_w);
    m->in_text = b.p<int32_t>((i64)B * S);
    m->in_target = b.p<int32_t>((i64)B * S);
    m->in_ctc = b.p<int32_t>((i64)B * S);
    m->in_ctc_len = b.p<int32_t>(B);
}

// ------------------------------------------------------------ the step --
struct Ctx {
    trba_model *m;
    cudaStream_t st;
    int B;
    float *P, *G;
    bool eval = false;  // inference: BN with the running statistics, no running-stat update
    const int8_t *nhwc_src = nullptr;  // the activations m->qh holds in NHWC order
};

struct ProbeScope {
    Probe *p = nullptr;
    cudaStream_t st;
    bool stamp = false;
    ProbeScope(trba_model *m, int kind, double ops, double bytes, cudaStream_t s) : st(s) {
        if (m->probe.kind != kind) return;
        p = &m->probe;
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        TRBA_CHECK(cudaStreamIsCapturing(st, &cs));
        stamp = cs == cudaStreamCaptureStatusActive;
        if (stamp) {
            if (p->nstamp + 2 > 2 * kProbeStamps) {
                p = nullptr;
                return;
            }
            stamp_kernel<<<1, 1, 0, st>>>(p->stamps + p->nstamp);
            TRBA_LAUNCH_CHECK();
            p->stamped = true;
        } else {
            while (p->ev.size() < p->used + 2) {
                cudaEvent_t e;
                TRBA_CHECK(cudaEventCreate(&e));
                p->ev.push_back(e);
            }
            TRBA_CHECK(cudaEventRecord(p->ev[p->used], st));
        }
        p->ops += ops;
        p->bytes += bytes;
        p->launches += 1;
    }
    ~ProbeScope() {
        if (!p) return;
        if (stamp) {
            stamp_kernel<<<1, 1, 0, st>>>(p->stamps + p->nstamp + 1);
            TRBA_LAUNCH_CHECK();
            p->nstamp += 2;
        } else {
            TRBA_CHECK(cudaEventRecord(p->ev[p->used + 1], st));
            p->used += 2;
        }
    }
};

void sgemm(Ctx &c, const seq::Gemm &g, cudaStream_t st) {
    ProbeScope ps(c.m, TRBA_PROBE_SGEMM, 2.0 * g.M * g.N * g.K, 4.0 * ((double)g.M * g.K + (double)g.K * g.N + (double)g.M * g.N),
                  st);
    seq::sgemm(g, st);
}

void conv_fwd(Ctx &c, ConvL &L, const int8_t *q_in, const float *s_in) {
    const int B = c.B;
    const i64 rows = L.rows(B);
    L.q_in = q_in;
    L.s_in = s_in;
    // Implicit GEMM: the forward writes no im2col matrix.  The weight
    // gradient's operand (the matrix itself for the reference-compatible
    // weight gradient, its transpose in the corrected mode) is built later,
    // off the forward path (wgrad_operands).
    if (L.implicit) {
        if (c.nhwc_src != q_in) {  // a downsample conv and conv1 share their input
            nhwc_from_nchw_i8(q_in, c.m->qh.get(), B, L.cin, L.H * L.W, c.st);
            c.nhwc_src = q_in;
        }
        // bytes: the int8 input + weights read, x (f32) written
        ProbeScope ps(c.m, TRBA_PROBE_CONV_GEMM, 2.0 * rows * L.cout * L.K,
                      (double)B * L.cin * L.H * L.W + (double)L.cout * L.K + 4.0 * rows * L.cout, c.st);
        const ConvGeo g{c.m->qh.get(), B, L.H, L.W, L.cin, L.kh, L.kw, L.sh, L.sw, L.ph, L.pw, L.Ho, L.Wo};
        if (!gemm_i8_conv_implicit_f32(g, L.wqh.get(), L.K, L.cout, L.x.get(), s_in, L.ws.get(),
                                       c.m->cfg.wq_per_channel != 0, L.bn_acc.get(), c.st))
            report_error(__FILE__, __LINE__, "conv forward implicit GEMM: unsupported operands", -1);
        return;
    }
    launch_im2col_pad(q_in, L.col.get(), B, L.cin, L.H, L.W, L.kh, L.kw, L.sh, L.sw, L.ph, L.pw, L.Ho, L.Wo, L.kp,
                      c.st);
    {
        // bytes: im2col operand + weights read, x (f32) written
        ProbeScope ps(c.m, TRBA_PROBE_CONV_GEMM, 2.0 * rows * L.cout * L.K,
                      (double)rows * L.kp + (double)L.cout * L.kp + 4.0 * rows * L.cout, c.st);
        if (!gemm_i8_conv_f32(L.col.get(), L.kp, L.wq.get(), L.kp, (int)rows, L.cout, L.K, L.x.get(), s_in,
                              L.ws.get(), c.m->cfg.wq_per_channel != 0, L.bn_acc.get(), L.Ho * L.Wo, c.st))
            report_error(__FILE__, __LINE__, "conv forward GEMM: operands not TMA-describable", -1);
    }
    if (c.m->cfg.wgrad_mode == 1 && !c.eval)  // the weight gradient's operand: training only
        qat::im2col_t(q_in, L.colT.get(), B, L.cin, L.H, L.W, L.kh, L.kw, L.sh, L.sw, L.ph, L.pw, L.Ho, L.Wo,
                      (int)a16l(rows), c.st);
}

// The weight-gradient operands of the implicit-GEMM convs (training), built
// from the inputs the forward kept (L.q_in) on the weight-gradient stream
// once the forward is done: they overlap the sequence head, whose
// recurrences leave most SMs idle, instead of the forward.  Last conv first,
// the order the backward needs them in; the weight-gradient stream runs them
// before the backward's weight-gradient work it queues behind them.
void wgrad_operands(Ctx &c) {
    trba_model *m = c.m;
    const bool correct = m->cfg.wgrad_mode == 1;
    bool forked = false;
    for (int i = (int)m->convs.size() - 1; i >= 0; --i) {
        ConvL &L = m->convs[i];
        if (!L.implicit) continue;
        if (!forked) {
            TRBA_CHECK(cudaEventRecord(m->fork_ev, c.st));
            TRBA_CHECK(cudaStreamWaitEvent(m->side, m->fork_ev, 0));
            forked = true;
        }
        const int B = c.B;
        if (correct)
            qat::im2col_t(L.q_in, L.colT.get(), B, L.cin, L.H, L.W, L.kh, L.kw, L.sh, L.sw, L.ph, L.pw, L.Ho, L.Wo,
                          (int)a16l(L.rows(B)), m->side);
        else
            launch_im2col_pad(L.q_in, L.col.get(), B, L.cin, L.H, L.W, L.kh, L.kw, L.sh, L.sw, L.ph, L.pw, L.Ho,
                              L.Wo, L.kp, m->side);
    }
}

qat::Src bn_src(Ctx &c, ConvL &L) {
    qat::Src s{};
    s.kind = c.eval ? qat::SRC_BN_EVAL : qat::SRC_BN;
    s.x = L.x.get();
    s.bn_acc = L.bn_acc.get();
    s.run_mean = L.run_mean.get();
    s.run_var = L.run_var.get();
    s.gamma = c.P + L.gamma_off;
    s.beta = c.P + L.beta_off;
    s.C = L.cout;
    s.HW = L.Ho * L.Wo;
    s.count = (i64)c.B * L.Ho * L.Wo;
    return s;
}

// conv + BN + (ReLU-)quantise: the reference's ConvQat::forward followed by
// relu_quant_owned (src/qnet.rs:788-916, 1102-1112).
void conv_bn_quant(Ctx &c, ConvL &L, const int8_t *q_in, const float *s_in) {
    conv_fwd(c, L, q_in, s_in);
    qat::Src s = bn_src(c, L);
    qat::act_stats(s, c.B, nullptr, L.mean.get(), L.var.get(), nullptr, L.ymax.get(), c.st);
    qat::act_quant(s, c.B, L.ymax.get(), L.s_q.get(), L.q.get(), true, c.st);
}

// Number of (input position, kernel tap) pairs along one axis whose output
// position lies on the output grid: the gather terms of the input gradient.
double valid_taps(int n_in, int k, int s, int pad, int n_out) {
    double v = 0.0;
    for (int i = 0; i < n_in; ++i)
        for (int t = 0; t < k; ++t) {
            const int q = i + pad - t;
            if (q >= 0 && q % s == 0 && q / s < n_out) v += 1.0;
        }
    return v;
}

// ConvQat::backward (src/qnet.rs:918-1083).  gi: input gradient (or null).
// gi: input gradient (or null).  gmax_scale / gmax_out (optional): the input
// gradient's max |gi * scale| for the block that consumes it, accumulated by
// the gather's epilogue instead of a separate pass.
void conv_bwd(Ctx &c, ConvL &L, const float *dy, const int8_t *mask_q, const float *add, float *gi,
              const float *gmax_scale = nullptr, float *gmax_out = nullptr) {
    const int B = c.B, HW = L.Ho * L.Wo;
    const i64 rows = L.rows(B), rp = a16l(rows);
    const bool compat = c.m->cfg.wgrad_mode == 0;
    cudaStream_t ws = c.m->side;
    // The input gradient of the reference reads the BN-output gradient dy
    // (not the BN-input gradient), so the BN backward chain and the weight
    // gradient feed nothing but the parameter gradients: they run on the
    // weight-gradient stream, joined once at the end of the backward pass,
    // while the chain of input gradients (the critical path) stays here.
    TRBA_CHECK(cudaEventRecord(c.m->fork_ev, c.st));
    TRBA_CHECK(cudaStreamWaitEvent(ws, c.m->fork_ev, 0));
    qat::bn_bwd_sums(dy, L.x.get(), L.mean.get(), L.var.get(), B, L.cout, HW, L.bwd_acc.get(), ws);
    qat::bn_dx_max(dy, L.x.get(), L.mean.get(), L.var.get(), c.P + L.gamma_off, L.bwd_acc.get(), B, L.cout, HW,
                   c.G + L.gamma_off, c.G + L.beta_off, L.dxmax.get(), ws);
    if (compat && (rows & 15)) TRBA_CHECK(cudaMemsetAsync(L.A.get(), 0, (size_t)a16(L.cout) * rp, ws));
    qat::bn_dx_quant(dy, L.x.get(), L.mean.get(), L.var.get(), c.P + L.gamma_off, L.bwd_acc.get(), B, L.cout, HW,
                     L.dxmax.get(), L.s_dx.get(), L.A.get(), compat ? (int)rows : (int)rp, compat, ws);
    const int splits = splitk_for(L.cout, L.K, (int)rows);
    const int8_t *Bop = compat ? L.col.get() : L.colT.get();
    {
        // bytes: quantised dx + im2col operand read, s32 dW accumulated
        ProbeScope ps(c.m, TRBA_PROBE_WGRAD_GEMM, 2.0 * rows * L.cout * L.K,
                      (double)rows * L.cout + (double)rows * L.kp + 4.0 * L.cout * L.K, ws);
        if (!gemm_i8_splitk_atomic(L.A.get(), (int)rp, Bop, (int)rp, L.gw.get(), L.cout, L.K, (int)rows, splits, ws))
            report_error(__FILE__, __LINE__, "conv wgrad GEMM: operands not TMA-describable", -1);
    }
    qat::grad_accum(L.gw.get(), L.s_dx.get(), L.s_in, (i64)L.cout * L.K, c.G + L.w_off, ws);
    if (gi) {
        // ops: one multiply and one add per (input element, valid tap, output channel)
        const double in_n = (double)B * L.cin * L.H * L.W;
        const double bytes = 4.0 * B * L.cout * HW + 4.0 * in_n + (mask_q ? in_n : 0.0) + (add ? 4.0 * in_n : 0.0) +
                             (double)L.cout * L.K;
        const double terms = (double)B * L.cin * L.cout * valid_taps(L.H, L.kh, L.sh, L.ph, L.Ho) *
                             valid_taps(L.W, L.kw, L.sw, L.pw, L.Wo);
        ProbeScope ps(c.m, TRBA_PROBE_DGRAD, 2.0 * terms, bytes, c.st);
        // per-channel scales are folded into the operands (dy per output
        // channel, or the exact gather's dequantised weights): final scale 1
        const bool pc = c.m->cfg.wq_per_channel != 0;
        if (L.tc_ok) {
            dgtc::Plan p = L.tc;
            dgtc::set_batch(p, B);
            dgtc::launch(p, L.wimg.get(), c.m->dg_planes.get(), dy, pc ? c.m->ones.get() : L.ws.get(), 1.0f,
                         pc ? L.ws.get() : nullptr,
                         mask_q, add, gi, gmax_scale, gmax_out, c.st);
            return;
        }
        qat::dgrad(dy, L.wT.get(), pc ? c.m->ones.get() : L.ws.get(), B, L.cin, L.H, L.W, L.cout, L.kh, L.kw, L.sh, L.sw, L.ph, L.pw, L.Ho,
                   L.Wo, L.cls_perm.empty() ? nullptr : L.d_perm.get(),
                   L.cls_perm.empty() ? nullptr : L.d_cstart.get(), (int)L.cls_start.size() - 1, mask_q, add, gi,
                   c.st, gmax_scale, gmax_out);
    }
}

// Joins the weight-gradient stream back into the step's stream.
void join_weight_grads(Ctx &c) {
    TRBA_CHECK(cudaEventRecord(c.m->join_ev, c.m->side));
    TRBA_CHECK(cudaStreamWaitEvent(c.st, c.m->join_ev, 0));
}

void cnn_forward(Ctx &c, const int8_t *img) {
    trba_model *m = c.m;
    auto &cv = m->convs;
    conv_bn_quant(c, cv[0], img, m->s_img.get());
    conv_bn_quant(c, cv[1], cv[0].q.get(), cv[0].s_q.get());
    launch_maxpool2x2_forward_i8(cv[1].q.get(), m->qpool.get(), c.B, cv[1].cout, cv[1].Ho, cv[1].Wo, c.st);
    const int8_t *q = m->qpool.get();
    const float *s = cv[1].s_q.get();
    for (auto &bl : m->blocks) {
        ConvL &c1 = cv[bl.c1], &c2 = cv[bl.c2];
        if (bl.ds >= 0) {
            ConvL &ds = cv[bl.ds];
            conv_fwd(c, ds, q, s);
            qat::act_stats(bn_src(c, ds), c.B, ds.y.get(), ds.mean.get(), ds.var.get(), nullptr, nullptr, c.st);
        }
        conv_bn_quant(c, c1, q, s);
        conv_fwd(c, c2, c1.q.get(), c1.s_q.get());
        qat::act_stats(bn_src(c, c2), c.B, c2.y.get(), c2.mean.get(), c2.var.get(), bl.pool.get(), nullptr, c.st);
        qat::se_forward(bl.pool.get(), c.P + bl.w1_off, c.P + bl.w2_off, c.B, bl.C, bl.R, bl.h1.get(), bl.gate.get(),
                        c.st);
        qat::Src z{};
        z.kind = bl.ds >= 0 ? qat::SRC_SE_RES_F : qat::SRC_SE_RES_Q;
        z.x = c2.y.get();
        z.gate = bl.gate.get();
        z.res_f = bl.ds >= 0 ? cv[bl.ds].y.get() : nullptr;
        z.res_q = q;
        z.res_s = s;
        z.C = bl.C;
        z.HW = bl.Ho * bl.Wo;
        qat::act_stats(z, c.B, nullptr, nullptr, nullptr, nullptr, bl.zmax.get(), c.st);
        qat::act_quant(z, c.B, bl.zmax.get(), bl.s_out.get(), bl.q_out.get(), true, c.st);
        q = bl.q_out.get();
        s = bl.s_out.get();
    }
    const int nc = (int)cv.size();
    conv_bn_quant(c, cv[nc - 2], q, s);
    conv_bn_quant(c, cv[nc - 1], cv[nc - 2].q.get(), cv[nc - 2].s_q.get());
    const ConvL &o1 = cv[nc - 1];
    qat::features(o1.q.get(), o1.s_q.get(), c.B, o1.cout, o1.Ho, o1.Wo, m->feat.get(), c.st);
    if (!c.eval) {
        bn_running_kernel<<<nc, 128, 0, c.st>>>(m->d_convtab, nc);
        TRBA_LAUNCH_CHECK();
    }
}

void cnn_backward(Ctx &c) {
    trba_model *m = c.m;
    auto &cv = m->convs;
    const int nc = (int)cv.size();
    ConvL &o0 = cv[nc - 2], &o1 = cv[nc - 1];
    qat::features_bwd(m->dfeat.get(), o1.q.get(), o1.s_q.get(), c.B, o1.cout, o1.Ho, o1.Wo, m->dy_o1.get(), c.st);
    conv_bwd(c, o1, m->dy_o1.get(), o0.q.get(), nullptr, m->dy_o0.get());
    // Each block's output gradient is re-quantised with max |gv * s_out|; the
    // gather that writes gv last accumulates that max in its epilogue.
    const int nb = (int)m->blocks.size();
    conv_bwd(c, o0, m->dy_o0.get(), nullptr, nullptr, m->gv_last.get(), nb ? m->blocks[nb - 1].s_out.get() : nullptr,
             nb ? m->blocks[nb - 1].gvmax.get() : nullptr);
    const float *gv = m->gv_last.get();
    for (int bi = nb - 1; bi >= 0; --bi) {
        BlockL &bl = m->blocks[bi];
        ConvL &c1 = cv[bl.c1], &c2 = cv[bl.c2];
        const float *next_scale = bi > 0 ? m->blocks[bi - 1].s_out.get() : nullptr;
        float *next_max = bi > 0 ? m->blocks[bi - 1].gvmax.get() : nullptr;
        qat::se_backward(gv, bl.s_out.get(), bl.gvmax.get(), bl.q_out.get(), bl.s_dq.get(), bl.dz.get(), c2.y.get(),
                         bl.gate.get(), bl.h1.get(), c.P + bl.w1_off, c.P + bl.w2_off, c.B, bl.C, bl.Ho * bl.Wo, bl.R,
                         bl.dpre1.get(), bl.dpre2.get(), bl.dpooled.get(), bl.dy2.get(), c.st);
        qat::se_weight_grads(bl.dpre1.get(), bl.dpre2.get(), bl.h1.get(), bl.pool.get(), c.B, bl.C, bl.R,
                             c.G + bl.w1_off, c.G + bl.w2_off, c.st);
        conv_bwd(c, c2, bl.dy2.get(), c1.q.get(), nullptr, bl.dy1.get());
        if (bl.ds >= 0) {
            conv_bwd(c, c1, bl.dy1.get(), nullptr, nullptr, bl.gin.get());
            // total = gi_in + dx_ds (src/qnet.rs:1345-1349)
            conv_bwd(c, cv[bl.ds], bl.dz.get(), nullptr, bl.gin.get(), bl.gin.get(), next_scale, next_max);
        } else {
            conv_bwd(c, c1, bl.dy1.get(), nullptr, bl.dz.get(), bl.gin.get(), next_scale, next_max);
        }
        gv = bl.gin.get();
    }
    qat::pool_bwd_mask(cv[1].q.get(), gv, cv[1].s_q.get(), c.B, cv[1].cout, cv[1].Ho, cv[1].Wo, m->dy_c1.get(), c.st);
    conv_bwd(c, cv[1], m->dy_c1.get(), cv[0].q.get(), nullptr, m->dy_c0.get());
    conv_bwd(c, cv[0], m->dy_c0.get(), nullptr, nullptr, nullptr);
    join_weight_grads(c);
}

seq::Gemm gemm(trba_model *m, int M, int N, int K, const float *A, i64 sam, i64 sak, const float *Bm, i64 sbk,
               i64 sbn, float *C, i64 ldc, bool accumulate = false, const float *bias = nullptr) {
    seq::Gemm g;
    g.M = M, g.N = N, g.K = K;
    g.A = A, g.sam = sam, g.sak = sak;
    g.B = Bm, g.sbk = sbk, g.sbn = sbn;
    g.C = C, g.ldc = ldc;
    g.accumulate = accumulate;
    g.bias = bias;
    g.ws = m->gemm_ws.get();
    g.ws_elems = m->gemm_ws_elems;
    return g;
}

void colsum(trba_model *m, const float *X, int rows, int cols, i64 ld, float *out, cudaStream_t st) {
    seq::col_sums(X, rows, cols, ld, m->ones.get(), out, true, m->gemm_ws.get(), m->gemm_ws_elems, st);
}

// Input projections of both directions, then both recurrences in one launch
// (independent: the directions share only the layer input).
void lstm_layer_fwd(Ctx &c, RnnL &r, const float *x) {
    trba_model *m = c.m;
    const int B = c.B, T = m->T, H = m->cfg.hidden;
    seq::LstmFwdDir dirs[2];
    for (int d = 0; d < 2; ++d) {
        sgemm(c, gemm(m, B * T, 4 * H, r.D, x, r.D, 1, c.P + r.wih[d], 1, r.D, r.xg[d].get(), 4 * H), c.st);
        dirs[d] = seq::LstmFwdDir{r.xg[d].get(), c.P + r.bih[d], c.P + r.bhh[d], c.P + r.whh[d], r.gates[d].get(),
                                  r.c[d].get(), r.hprev[d].get(), d, d};
    }
    seq::lstm_fwd(dirs, 2, B, T, H, r.cat.get(), c.st);
}

void head_forward(Ctx &c, const int32_t *text_in, const int32_t *target, const int32_t *ctc_tgt,
                  const int32_t *ctc_len) {
    trba_model *m = c.m;
    const auto &cf = m->cfg;
    const int B = c.B, T = m->T, H = cf.hidden, V = cf.classes, S = m->steps;
    const float *x = m->feat.get();
    for (auto &r : m->rnn) {  // BiLstmLayer::forward (src/rnn.rs:167-174)
        lstm_layer_fwd(c, r, x);
        sgemm(c, gemm(m, B * T, H, 2 * H, r.cat.get(), 2 * H, 1, c.P + r.pw, 1, 2 * H, r.y.get(), H, false, c.P + r.pb),
                   c.st);
        x = r.y.get();
    }
    const float *enc = x;  // [B, T, H]
    const i64 oi2h = entry_off(m, "attn.i2h.w");
    sgemm(c, gemm(m, B * T, H, H, enc, H, 1, c.P + oi2h, 1, H, m->proj_h.get(), H), c.st);
    seq::AttnFwd a{};
    a.bh = enc;
    a.proj_h = m->proj_h.get();
    a.text_in = text_in;
    a.h2h_w = c.P + entry_off(m, "attn.h2h.w");
    a.h2h_b = c.P + entry_off(m, "attn.h2h.b");
    a.score_w = c.P + entry_off(m, "attn.score.w");
    a.w_ih = c.P + entry_off(m, "attn.w_ih");
    a.b_ih = c.P + entry_off(m, "attn.b_ih");
    a.w_hh = c.P + entry_off(m, "attn.w_hh");
    a.b_hh = c.P + entry_off(m, "attn.b_hh");
    a.B = B, a.T = T, a.H = H, a.V = V, a.steps = S;
    a.tanh_tr = m->tanh_tr.get();
    a.alpha = m->alpha.get();
    a.cell_in = m->cell_in.get();
    a.gates = m->agates.get();
    a.hs = m->hs.get();
    a.cs = m->cs.get();
    seq::attn_fwd(a, c.st);
    sgemm(c, gemm(m, S * B, V, H, m->hs.get(), H, 1, c.P + entry_off(m, "attn.gen.w"), 1, H, m->logits.get(), V, 0.0f,
                    c.P + entry_off(m, "attn.gen.b")),
               c.st);
    sgemm(c, gemm(m, B * T, V, H, enc, H, 1, c.P + entry_off(m, "ctc.w"), 1, H, m->ctc_logits.get(), V, 0.0f,
                    c.P + entry_off(m, "ctc.b")),
               c.st);
    seq::ce_rows(m->logits.get(), target, B, S, V, cf.pad, m->dlogits.get(), m->row_loss.get(), c.st);
    seq::ctc(m->ctc_logits.get(), ctc_tgt, ctc_len, S, B, T, V, cf.ctc_weight, m->dctc.get(),
             m->ctc_sample_loss.get(), c.st);
    seq::loss_finalize(m->row_loss.get(), target, B, S, cf.pad, m->ctc_sample_loss.get(), ctc_len, T, cf.ctc_weight,
                       m->dlogits.get(), V, m->loss.get(), c.st);
}

// Inference head (run_inference, later snapshot src/main.rs:2690): the
// BiLSTM stack as in training, then greedy attention decoding.
void head_infer(Ctx &c, int32_t *step_tokens) {
    trba_model *m = c.m;
    const auto &cf = m->cfg;
    const int B = c.B, T = m->T, H = cf.hidden, V = cf.classes, S = m->steps;
    const float *x = m->feat.get();
    for (auto &r : m->rnn) {
        lstm_layer_fwd(c, r, x);
        sgemm(c, gemm(m, B * T, H, 2 * H, r.cat.get(), 2 * H, 1, c.P + r.pw, 1, 2 * H, r.y.get(), H, false, c.P + r.pb),
              c.st);
        x = r.y.get();
    }
    const float *enc = x;
    sgemm(c, gemm(m, B * T, H, H, enc, H, 1, c.P + entry_off(m, "attn.i2h.w"), 1, H, m->proj_h.get(), H), c.st);
    seq::AttnFwd a{};
    a.bh = enc;
    a.proj_h = m->proj_h.get();
    a.h2h_w = c.P + entry_off(m, "attn.h2h.w");
    a.h2h_b = c.P + entry_off(m, "attn.h2h.b");
    a.score_w = c.P + entry_off(m, "attn.score.w");
    a.w_ih = c.P + entry_off(m, "attn.w_ih");
    a.b_ih = c.P + entry_off(m, "attn.b_ih");
    a.w_hh = c.P + entry_off(m, "attn.w_hh");
    a.b_hh = c.P + entry_off(m, "attn.b_hh");
    a.gen_w = c.P + entry_off(m, "attn.gen.w");
    a.gen_b = c.P + entry_off(m, "attn.gen.b");
    a.sos = cf.sos;
    a.B = B, a.T = T, a.H = H, a.V = V, a.steps = S;
    a.step_tokens = step_tokens;
    seq::attn_decode(a, c.st);
}

void head_backward(Ctx &c) {
    trba_model *m = c.m;
    const auto &cf = m->cfg;
    const int B = c.B, T = m->T, H = cf.hidden, V = cf.classes, S = m->steps, R = S * B;
    const float *enc = m->rnn.back().y.get();
    const i64 ogw = entry_off(m, "attn.gen.w"), ogb = entry_off(m, "attn.gen.b");
    // generator (src/attn.rs:274-284)
    sgemm(c, gemm(m, V, H, R, m->dlogits.get(), 1, V, m->hs.get(), H, 1, c.G + ogw, H, true), c.st);
    colsum(m, m->dlogits.get(), R, V, V, c.G + ogb, c.st);
    sgemm(c, gemm(m, R, H, V, m->dlogits.get(), V, 1, c.P + ogw, H, 1, m->d_out_hid.get(), H), c.st);
    seq::AttnBwd a{};
    a.d_out_hid = m->d_out_hid.get();
    a.bh = enc;
    a.tanh_tr = m->tanh_tr.get();
    a.alpha = m->alpha.get();
    a.gates = m->agates.get();
    a.cs = m->cs.get();
    a.score_w = c.P + entry_off(m, "attn.score.w");
    a.w_ih = c.P + entry_off(m, "attn.w_ih");
    a.w_hh = c.P + entry_off(m, "attn.w_hh");
    a.h2h_w = c.P + entry_off(m, "attn.h2h.w");
    a.B = B, a.T = T, a.H = H, a.V = V, a.steps = S;
    a.dgates = m->adg.get();
    a.de = m->ade.get();
    a.dprojhh = m->adprojhh.get();
    a.d_proj_h = m->d_proj_h.get();
    a.d_bh = m->d_bh.get();
    seq::attn_bwd(a, c.st);
    const int CV = H + V;
    float *dg = m->adg.get();
    sgemm(c, gemm(m, 4 * H, CV, R, dg, 1, 4 * H, m->cell_in.get(), CV, 1, c.G + entry_off(m, "attn.w_ih"), CV, true),
               c.st);
    colsum(m, dg, R, 4 * H, 4 * H, c.G + entry_off(m, "attn.b_ih"), c.st);
    colsum(m, dg, R, 4 * H, 4 * H, c.G + entry_off(m, "attn.b_hh"), c.st);
    // w_hh and h2h: h_prev of step st is hs of st-1 (zero at st = 0)
    sgemm(c, gemm(m, 4 * H, H, R - B, dg + (i64)B * 4 * H, 1, 4 * H, m->hs.get(), H, 1,
                    c.G + entry_off(m, "attn.w_hh"), H, true),
               c.st);
    sgemm(c, gemm(m, H, H, R - B, m->adprojhh.get() + (i64)B * H, 1, H, m->hs.get(), H, 1,
                    c.G + entry_off(m, "attn.h2h.w"), H, true),
               c.st);
    colsum(m, m->adprojhh.get(), R, H, H, c.G + entry_off(m, "attn.h2h.b"), c.st);
    sgemm(c, gemm(m, 1, H, R * T, m->ade.get(), 0, 1, m->tanh_tr.get(), H, 1, c.G + entry_off(m, "attn.score.w"), H,
                    true),
               c.st);
    const i64 oi2h = entry_off(m, "attn.i2h.w");
    sgemm(c, gemm(m, H, H, B * T, m->d_proj_h.get(), 1, H, enc, H, 1, c.G + oi2h, H, true), c.st);
    sgemm(c, gemm(m, B * T, H, H, m->d_proj_h.get(), H, 1, c.P + oi2h, H, 1, m->d_bh.get(), H, true), c.st);
    // CTC head (src/main.rs:2344): LinearF backward
    const i64 ocw = entry_off(m, "ctc.w"), ocb = entry_off(m, "ctc.b");
    sgemm(c, gemm(m, V, H, B * T, m->dctc.get(), 1, V, enc, H, 1, c.G + ocw, H, true), c.st);
    colsum(m, m->dctc.get(), B * T, V, V, c.G + ocb, c.st);
    sgemm(c, gemm(m, B * T, H, V, m->dctc.get(), V, 1, c.P + ocw, H, 1, m->d_bh.get(), H, true), c.st);
    // BiLSTM backward, top layer first (src/rnn.rs:176-198)
    const float *dy = m->d_bh.get();
    for (int li = (int)m->rnn.size() - 1; li >= 0; --li) {
        RnnL &r = m->rnn[li];
        const float *xin = li == 0 ? m->feat.get() : m->rnn[li - 1].y.get();
        sgemm(c, gemm(m, H, 2 * H, B * T, dy, 1, H, r.cat.get(), 2 * H, 1, c.G + r.pw, 2 * H, true), c.st);
        colsum(m, dy, B * T, H, H, c.G + r.pb, c.st);
        sgemm(c, gemm(m, B * T, 2 * H, H, dy, H, 1, c.P + r.pw, 2 * H, 1, r.dcat.get(), 2 * H), c.st);
        float *dxout = li == 0 ? m->dfeat.get() : r.dx.get();
        seq::LstmBwdDir bdirs[2];
        for (int d = 0; d < 2; ++d)
            bdirs[d] = seq::LstmBwdDir{r.gates[d].get(), r.c[d].get(), c.P + r.whh[d], r.dg[d].get(), d, d};
        seq::lstm_bwd(bdirs, 2, r.dcat.get(), B, T, H, c.st);
        for (int d = 0; d < 2; ++d) {
            const float *g = r.dg[d].get();
            sgemm(c, gemm(m, 4 * H, r.D, B * T, g, 1, 4 * H, xin, r.D, 1, c.G + r.wih[d], r.D, true), c.st);
            sgemm(c, gemm(m, 4 * H, H, B * T, g, 1, 4 * H, r.hprev[d].get(), H, 1, c.G + r.whh[d], H, true), c.st);
            colsum(m, g, B * T, 4 * H, 4 * H, c.G + r.bih[d], c.st);
            colsum(m, g, B * T, 4 * H, 4 * H, c.G + r.bhh[d], c.st);
            sgemm(c, gemm(m, B * T, r.D, 4 * H, g, 4 * H, 1, c.P + r.wih[d], r.D, 1, dxout, r.D, d != 0),
                       c.st);
        }
        dy = dxout;
    }
}

// max |w| per conv, or per output channel, into m->wmax_bits.
void launch_wmax(trba_model *m, const float *P, cudaStream_t st) {
    const int ncv = (int)m->conv_segs.size();
    if (m->cfg.wq_per_channel) {
        conv_wmax_rows_kernel<<<dim3(4, ncv), 256, 0, st>>>(m->d_conv, P, m->wmax_bits.get());
    } else {
        TRBA_CHECK(cudaMemsetAsync(m->wmax_bits.get(), 0, sizeof(unsigned) * m->n_chan, st));
        conv_wmax_kernel<<<dim3(16, ncv), 256, 0, st>>>(m->d_conv, P, m->wmax_bits.get());
    }
    TRBA_LAUNCH_CHECK();
}

void optimizer(trba_model *m, cudaStream_t st) {
    const auto &cf = m->cfg;
    float *P = m->P.get(), *G = m->G.get();
    sumsq_kernel<<<grid_for(m->n_params), 256, 0, st>>>(G, m->n_params, m->gsq_total.get());
    step_state_kernel<<<1, 32, 0, st>>>(m->step_state.get(), cf.clip_warmup);
    clip_factor_kernel<<<1, 32, 0, st>>>(m->gsq_total.get(), m->step_state.get(), m->clip_f.get());
    m->t += 1;  // host mirror of step_state[0]
    const double lr = (double)cf.lr, wd = (double)cf.weight_decay;
    const int nv = (int)m->vec_segs.size(), nm = (int)m->mat_segs.size(), ncv = (int)m->conv_segs.size();
    adam_segs_kernel<<<dim3(4, nv), 256, 0, st>>>(m->d_vec, P, G, m->Mm.get(), m->Vv.get(), m->clip_f.get(), lr, wd,
                                                  (double)0.9f, (double)0.999f, (double)1e-8f,
                                                  m->step_state.get());
    muon_mat_norm_kernel<<<nm, 256, 0, st>>>(m->d_mat, G, m->clip_f.get(), cf.lr, cf.muon_cap, m->mat_step.get());
    muon_mat_apply_kernel<<<dim3(8, nm), 256, 0, st>>>(m->d_mat, P, G, m->clip_f.get(), m->mat_step.get(),
                                                       1.0f - cf.lr * cf.weight_decay);
    conv_gsq_kernel<<<dim3(8, ncv), 256, 0, st>>>(m->d_conv, G, m->conv_gsq.get());
    conv_muon_apply_kernel<<<dim3(16, ncv), 256, 0, st>>>(m->d_conv, P, G, m->conv_gsq.get(), m->clip_f.get(), lr, wd,
                                                          (double)cf.muon_cap);
    launch_wmax(m, P, st);
    conv_quant_kernel<<<dim3(16, ncv), 256, 0, st>>>(m->d_conv, P, m->d_convtab, m->wmax_bits.get());
    TRBA_LAUNCH_CHECK();
}

void requantize(trba_model *m, cudaStream_t st) {
    const int ncv = (int)m->conv_segs.size();
    launch_wmax(m, m->P.get(), st);
    conv_quant_kernel<<<dim3(16, ncv), 256, 0, st>>>(m->d_conv, m->P.get(), m->d_convtab, m->wmax_bits.get());
    TRBA_LAUNCH_CHECK();
}

template <typename T>
T *upload_table(const std::vector<T> &v) {
    T *d = nullptr;
    if (v.empty()) return nullptr;
    TRBA_CHECK(cudaMalloc(&d, sizeof(T) * v.size()));
    TRBA_CHECK(cudaMemcpy(d, v.data(), sizeof(T) * v.size(), cudaMemcpyHostToDevice));
    return d;
}

int training_refused(trba_model *) {
    report_error(__FILE__, __LINE__, "inference-only model: training entry points are not available", -1);
    return -3;
}

int cuda_status() {
    const int e = trba_last_error();
    return e > 0 ? e : (e < 0 ? -e : 0);
}

}  // namespace

extern "C" {

void trba_model_default_config(trba_model_config *c) {
    std::memset(c, 0, sizeof(*c));
    c->fd = 128;
    c->hidden = 64;
    c->classes = 130;
    c->img_h = 32;
    c->img_w = 160;
    c->max_len = 20;
    c->rnn_layers = 2;
    c->batch = 48;
    c->sos = 1;
    c->eos = 2;
    c->pad = 0;
    c->lr = 5.107e-4f;
    c->weight_decay = 1.9548e-5f;
    c->ctc_weight = 0.03f;
    c->muon_cap = 10.0f;
    c->clip_warmup = 500;
    c->wgrad_mode = 0;
    c->dgrad_mode = 0;
    c->wq_per_channel = 0;
    c->inference_only = 0;
    c->conv_fwd_mode = 1;
}

trba_model *trba_model_create(const trba_model_config *cfg) {
    if (!cfg || cfg->fd < 16 || cfg->fd % 16 || cfg->fd > 512 || cfg->batch <= 0 || cfg->hidden <= 0 ||
        cfg->hidden > 128 || cfg->hidden % 8 || cfg->classes <= 3 || cfg->img_h < 8 || cfg->img_w < 8 || (cfg->img_h & 1) ||
        (cfg->img_w & 1) || cfg->max_len <= 0 || cfg->rnn_layers <= 0 || cfg->wgrad_mode < 0 ||
        cfg->wgrad_mode > 1 || cfg->dgrad_mode < 0 || cfg->dgrad_mode > 1 ||
        cfg->wq_per_channel < 0 || cfg->wq_per_channel > 1 || cfg->inference_only < 0 || cfg->inference_only > 1 ||
        cfg->conv_fwd_mode < 0 || cfg->conv_fwd_mode > 1) {
        report_error(__FILE__, __LINE__, "trba_model_create: unsupported configuration", -1);
        return nullptr;
    }
    trba_model *m = new trba_model();
    m->cfg = *cfg;
    m->B = cfg->batch;
    plan(m);
    if (m->T <= 0 || m->Hf <= 0) {
        report_error(__FILE__, __LINE__, "trba_model_create: image too small for the backbone", -1);
        delete m;
        return nullptr;
    }
    allocate(m);
    TRBA_CHECK(cudaMalloc(&m->arena.base, m->arena.used));
    TRBA_CHECK(cudaMalloc(&m->zarena.base, m->zarena.used));
    TRBA_CHECK(cudaMemset(m->arena.base, 0, m->arena.used));
    TRBA_CHECK(cudaMemset(m->zarena.base, 0, m->zarena.used));
    const float s_img = 1.0f / 127.0f;  // src/main.rs:1997
    TRBA_CHECK(cudaMemcpy(m->s_img.get(), &s_img, 4, cudaMemcpyHostToDevice));
    std::vector<trba_model::ConvTab> tab;
    for (auto &L : m->convs) {
        tab.push_back({L.wq.get(), L.ws.get(), L.wmax.get(), L.mean.get(), L.var.get(), L.run_mean.get(),
                       L.run_var.get(), L.cout, L.K, L.kp, L.tc_ok ? nullptr : L.wT.get(), L.kh * L.kw,
                       L.d_tc.get(), L.wimg.get(), m->cfg.wq_per_channel, L.implicit ? L.wqh.get() : nullptr});
        // (the input-gradient tables are training buffers: absent in an inference-only model)
        if (L.d_tc.get()) TRBA_CHECK(cudaMemcpy(L.d_tc.get(), &L.tc, sizeof(dgtc::Plan), cudaMemcpyHostToDevice));
        if (L.d_perm.get() && !L.cls_perm.empty()) {
            TRBA_CHECK(cudaMemcpy(L.d_perm.get(), L.cls_perm.data(), sizeof(int) * L.cls_perm.size(),
                                  cudaMemcpyHostToDevice));
            TRBA_CHECK(cudaMemcpy(L.d_cstart.get(), L.cls_start.data(), sizeof(int) * L.cls_start.size(),
                                  cudaMemcpyHostToDevice));
        }
        fill_f32_kernel<<<1, 128>>>(L.run_var.get(), L.cout, true);
    }
    m->d_convtab = upload_table(tab);
    m->d_vec = upload_table(m->vec_segs);
    m->d_mat = upload_table(m->mat_segs);
    m->d_conv = upload_table(m->conv_segs);
    {
        const i64 n1 = (i64)m->B * (m->steps > m->T ? m->steps : m->T);
        fill_f32_kernel<<<grid_for(n1), 256>>>(m->ones.get(), n1, 1.0f);
    }
    TRBA_CHECK(cudaEventCreateWithFlags(&m->ev, cudaEventDisableTiming));
    {
        // The replayed step's stream (the chain of input gradients is its
        // critical path) at the highest priority, the weight-gradient stream
        // at the lowest: when both have CTAs waiting, the critical chain's are
        // placed first and the weight gradients fill the SMs it leaves free.
        int least = 0, greatest = 0;
        TRBA_CHECK(cudaDeviceGetStreamPriorityRange(&least, &greatest));
        TRBA_CHECK(cudaStreamCreateWithPriority(&m->side, cudaStreamNonBlocking, least));
        TRBA_CHECK(cudaStreamCreateWithPriority(&m->gstream, cudaStreamNonBlocking, greatest));
    }
    TRBA_CHECK(cudaMalloc(&m->probe.stamps, 2 * kProbeStamps * sizeof(unsigned long long)));
    TRBA_CHECK(cudaEventCreateWithFlags(&m->gfork, cudaEventDisableTiming));
    TRBA_CHECK(cudaEventCreateWithFlags(&m->gjoin, cudaEventDisableTiming));
    TRBA_CHECK(cudaEventCreateWithFlags(&m->fork_ev, cudaEventDisableTiming));
    TRBA_CHECK(cudaEventCreateWithFlags(&m->join_ev, cudaEventDisableTiming));
    TRBA_CHECK(cudaDeviceSynchronize());
    return m;
}

void trba_model_destroy(trba_model *m) {
    if (!m) return;
    if (m->comm) nccl().CommDestroy(m->comm);
    cudaFree(m->arena.base);
    cudaFree(m->zarena.base);
    cudaFree(m->d_convtab);
    cudaFree(m->d_vec);
    cudaFree(m->d_mat);
    cudaFree(m->d_conv);
    if (m->ev) cudaEventDestroy(m->ev);
    if (m->fork_ev) cudaEventDestroy(m->fork_ev);
    if (m->join_ev) cudaEventDestroy(m->join_ev);
    if (m->side) cudaStreamDestroy(m->side);
    if (m->gexec) cudaGraphExecDestroy(m->gexec);
    if (m->gfork) cudaEventDestroy(m->gfork);
    if (m->gjoin) cudaEventDestroy(m->gjoin);
    if (m->gstream) cudaStreamDestroy(m->gstream);
    for (cudaEvent_t e : m->probe.ev) cudaEventDestroy(e);
    if (m->probe.stamps) cudaFree(m->probe.stamps);
    delete m;
}

long long trba_model_param_count(const trba_model *m) { return m ? m->n_params : -1; }
int trba_model_param_entries(const trba_model *m) { return m ? (int)m->manifest.size() : -1; }

int trba_model_param_entry(const trba_model *m, int i, char *name, int name_cap, long long *offset, int *rows,
                           int *cols, int *kind) {
    if (!m || i < 0 || i >= (int)m->manifest.size()) return -1;
    const Entry &e = m->manifest[i];
    if (name && name_cap > 0) {
        std::strncpy(name, e.name.c_str(), name_cap - 1);
        name[name_cap - 1] = 0;
    }
    if (offset) *offset = e.off;
    if (rows) *rows = e.rows;
    if (cols) *cols = e.cols;
    if (kind) *kind = e.kind;
    return 0;
}

int trba_model_set_params(trba_model *m, const float *host, long long n) {
    if (!m || !host || n != m->n_params) return -1;
    TRBA_CHECK(cudaMemcpy(m->P.get(), host, n * 4, cudaMemcpyHostToDevice));
    if (!m->cfg.inference_only) {
        TRBA_CHECK(cudaMemset(m->Mm.get(), 0, n * 4));
        TRBA_CHECK(cudaMemset(m->Vv.get(), 0, n * 4));
    }
    m->t = 0;
    TRBA_CHECK(cudaMemset(m->step_state.get(), 0, 4 * sizeof(double)));
    requantize(m, 0);
    TRBA_CHECK(cudaDeviceSynchronize());
    return cuda_status();
}

int trba_model_get_params(trba_model *m, float *host, long long n) {
    if (!m || !host || n != m->n_params) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    TRBA_CHECK(cudaMemcpy(host, m->P.get(), n * 4, cudaMemcpyDeviceToHost));
    return cuda_status();
}

int trba_model_get_grads(trba_model *m, float *host, long long n) {
    if (m && m->cfg.inference_only) return training_refused(m);
    if (!m || !host || n != m->n_params) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    TRBA_CHECK(cudaMemcpy(host, m->G.get(), n * 4, cudaMemcpyDeviceToHost));
    return cuda_status();
}

float *trba_model_grad_buffer(trba_model *m) { return m ? m->G.get() : nullptr; }
const float *trba_model_loss_dev(const trba_model *m) { return m ? m->loss.get() : nullptr; }
const int32_t *trba_model_step_tokens_dev(const trba_model *m) { return m ? m->step_tokens.get() : nullptr; }
long long trba_model_step_count(const trba_model *m) { return m ? m->t : -1; }
long long trba_model_device_bytes(const trba_model *m) {
    return m ? (long long)(m->arena.used + m->zarena.used) : -1;
}

long long trba_model_running_stats_count(const trba_model *m) {
    if (!m) return -1;
    long long n = 0;
    for (auto &L : m->convs) n += 2 * L.cout;
    return n;
}

int trba_model_get_running_stats(trba_model *m, float *host, long long n) {
    if (!m || !host || n != trba_model_running_stats_count(m)) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    long long o = 0;
    for (auto &L : m->convs) {
        TRBA_CHECK(cudaMemcpy(host + o, L.run_mean.get(), L.cout * 4, cudaMemcpyDeviceToHost));
        TRBA_CHECK(cudaMemcpy(host + o + L.cout, L.run_var.get(), L.cout * 4, cudaMemcpyDeviceToHost));
        o += 2 * L.cout;
    }
    return cuda_status();
}

int trba_model_forward_backward(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
                                const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, void *stream) {
    if (!m || !img || !text_in || !target || !ctc_tgt || !ctc_len || batch <= 0 || batch > m->B) return -1;
    if (m->cfg.inference_only) return training_refused(m);
    cudaStream_t st = as_stream(stream);
    Ctx c{m, st, batch, m->P.get(), m->G.get()};
    m->last_B = batch;
    if (m->probe.kind >= 0) m->probe.steps += 1;
    TRBA_CHECK(cudaMemsetAsync(m->zarena.base, 0, m->zarena.used, st));
    TRBA_CHECK(cudaMemsetAsync(m->G.get(), 0, (size_t)m->n_params * 4, st));
    {
        ProbeScope ps(m, TRBA_PROBE_PHASE_CNN_FWD, 0.0, 0.0, st);
        cnn_forward(c, img);
    }
    wgrad_operands(c);
    {
        ProbeScope ps(m, TRBA_PROBE_PHASE_HEAD_FWD, 0.0, 0.0, st);
        head_forward(c, text_in, target, ctc_tgt, ctc_len);
    }
    {
        ProbeScope ps(m, TRBA_PROBE_PHASE_HEAD_BWD, 0.0, 0.0, st);
        head_backward(c);
    }
    {
        ProbeScope ps(m, TRBA_PROBE_PHASE_CNN_BWD, 0.0, 0.0, st);
        cnn_backward(c);
    }
    return cuda_status();
}

int trba_model_infer(trba_model *m, const int8_t *img, int batch, int32_t *step_tokens, void *stream) {
    if (!m || !img || batch <= 0 || batch > m->B) return -1;
    cudaStream_t st = as_stream(stream);
    Ctx c{m, st, batch, m->P.get(), m->G.get()};
    c.eval = true;
    m->last_B = batch;
    // the per-tensor max-abs scalars (and BN sums) accumulate into the zeroed arena
    TRBA_CHECK(cudaMemsetAsync(m->zarena.base, 0, m->zarena.used, st));
    cnn_forward(c, img);
    head_infer(c, step_tokens ? step_tokens : m->step_tokens.get());
    return cuda_status();
}

int trba_model_infer_host(trba_model *m, const int8_t *img, int batch, int32_t *tokens, int32_t *lengths,
                          void *stream) {
    if (!m || !img || !tokens || !lengths || batch <= 0 || batch > m->B) return -1;
    cudaStream_t st = as_stream(stream);
    const auto &cf = m->cfg;
    const int S = m->steps;
    TRBA_CHECK(cudaMemcpyAsync(m->in_img.get(), img, (size_t)batch * 3 * cf.img_h * cf.img_w, cudaMemcpyHostToDevice,
                               st));
    int rc = trba_model_infer(m, m->in_img.get(), batch, nullptr, stream);
    if (rc) return rc;
    std::vector<int32_t> stok((size_t)S * batch);
    TRBA_CHECK(cudaMemcpyAsync(stok.data(), m->step_tokens.get(), stok.size() * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, st));
    TRBA_CHECK(cudaStreamSynchronize(st));
    // src/attn.rs:423-443: eos is not emitted; decoding stops after the first
    // step at which every sample of the batch produced eos.
    int last = S - 1;
    for (int s = 0; s < S; ++s) {
        bool all_eos = true;
        for (int b = 0; b < batch && all_eos; ++b) all_eos = stok[(size_t)s * batch + b] == cf.eos;
        if (all_eos) {
            last = s;
            break;
        }
    }
    for (int b = 0; b < batch; ++b) {
        int n = 0;
        for (int s = 0; s <= last; ++s) {
            const int t = stok[(size_t)s * batch + b];
            if (t != cf.eos) tokens[(size_t)b * S + n++] = t;
        }
        lengths[b] = n;
        for (int j = n; j < S; ++j) tokens[(size_t)b * S + j] = -1;
    }
    return cuda_status();
}

int trba_model_optimizer_step(trba_model *m, void *stream) {
    if (!m) return -1;
    if (m->cfg.inference_only) return training_refused(m);
    optimizer(m, as_stream(stream));
    return cuda_status();
}

}  // extern "C"

namespace {

// forward_backward, the data-parallel gradient all-reduce, optimizer_step.
int step_body(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
              const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, cudaStream_t st) {
    int rc = trba_model_forward_backward(m, img, text_in, target, ctc_tgt, ctc_len, batch, st);
    if (rc) return rc;
    ProbeScope ps(m, TRBA_PROBE_PHASE_OPTIMIZER, 0.0, 0.0, st);
    if (m->comm) {
        const ncclResult_t r = nccl().AllReduce(m->G.get(), m->G.get(), (size_t)m->n_params, ncclFloat, ncclAvg,
                                                m->comm, st);
        if (r != ncclSuccess) {
            report_error(__FILE__, __LINE__, nccl().GetErrorString(r), (int)r);
            return (int)r;
        }
    }
    return trba_model_optimizer_step(m, st);
}

// The step as one CUDA graph: recorded on the model's own stream the first
// time these input pointers and batch are seen (recording executes nothing),
// then replayed; the caller's stream is joined in and out with events.
int graph_step(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
               const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, cudaStream_t user) {
    const void *key[5] = {img, text_in, target, ctc_tgt, ctc_len};
    bool same = m->gexec && m->gkey_batch == batch && m->gkey_probe == m->probe.kind;
    for (int i = 0; i < 5 && same; ++i) same = m->gkey[i] == key[i];
    if (!same) {
        if (m->gexec) {
            TRBA_CHECK(cudaGraphExecDestroy(m->gexec));
            m->gexec = nullptr;
        }
        const long long t_host = m->t, l0 = launches_so_far();
        cudaGraph_t g = nullptr;
        TRBA_CHECK(cudaStreamBeginCapture(m->gstream, cudaStreamCaptureModeRelaxed));
        const int rc = step_body(m, img, text_in, target, ctc_tgt, ctc_len, batch, m->gstream);
        const cudaError_t e = cudaStreamEndCapture(m->gstream, &g);
        m->t = t_host;  // recording ran nothing
        m->graph_kernels = launches_so_far() - l0;
        count_launches(-m->graph_kernels);  // counted when replayed
        if (rc || e != cudaSuccess || !g) {
            if (g) cudaGraphDestroy(g);
            report_error(__FILE__, __LINE__, "trba_model_train_step: recording the step graph failed",
                         e != cudaSuccess ? (int)e : -1);
            return rc ? rc : -1;
        }
        const cudaError_t ei = cudaGraphInstantiate(&m->gexec, g, 0);
        cudaGraphDestroy(g);
        if (ei != cudaSuccess) {
            m->gexec = nullptr;
            report_error(__FILE__, __LINE__, "trba_model_train_step: instantiating the step graph failed", (int)ei);
            return (int)ei;
        }
        for (int i = 0; i < 5; ++i) m->gkey[i] = key[i];
        m->gkey_batch = batch;
        m->gkey_probe = m->probe.kind;
        m->last_B = batch;
    }
    TRBA_CHECK(cudaEventRecord(m->gfork, user));
    TRBA_CHECK(cudaStreamWaitEvent(m->gstream, m->gfork, 0));
    TRBA_CHECK(cudaGraphLaunch(m->gexec, m->gstream));
    count_launches(m->graph_kernels);
    TRBA_CHECK(cudaEventRecord(m->gjoin, m->gstream));
    TRBA_CHECK(cudaStreamWaitEvent(user, m->gjoin, 0));
    m->t += 1;
    return cuda_status();
}

}  // namespace

extern "C" {

int trba_model_train_step(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
                          const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, void *stream) {
    if (!m || !img || !text_in || !target || !ctc_tgt || !ctc_len || batch <= 0 || batch > m->B) return -1;
    if (m->cfg.inference_only) return training_refused(m);
    if (m->use_graphs)
        return graph_step(m, img, text_in, target, ctc_tgt, ctc_len, batch, as_stream(stream));
    return step_body(m, img, text_in, target, ctc_tgt, ctc_len, batch, as_stream(stream));
}

int trba_model_use_graphs(trba_model *m, int enable) {
    if (!m) return -1;
    m->use_graphs = enable != 0;
    if (!m->use_graphs && m->gexec) {
        TRBA_CHECK(cudaGraphExecDestroy(m->gexec));
        m->gexec = nullptr;
    }
    return cuda_status();
}

int trba_model_train_step_host(trba_model *m, const int8_t *img, const int32_t *text_in, const int32_t *target,
                               const int32_t *ctc_tgt, const int32_t *ctc_len, int batch, float *loss_host,
                               void *stream) {
    if (!m || batch <= 0 || batch > m->B || !loss_host) return -1;
    if (m->cfg.inference_only) return training_refused(m);
    cudaStream_t st = as_stream(stream);
    const auto &cf = m->cfg;
    const size_t S = (size_t)m->steps;
    TRBA_CHECK(cudaMemcpyAsync(m->in_img.get(), img, (size_t)batch * 3 * cf.img_h * cf.img_w, cudaMemcpyHostToDevice, st));
    TRBA_CHECK(cudaMemcpyAsync(m->in_text.get(), text_in, batch * S * 4, cudaMemcpyHostToDevice, st));
    TRBA_CHECK(cudaMemcpyAsync(m->in_target.get(), target, batch * S * 4, cudaMemcpyHostToDevice, st));
    TRBA_CHECK(cudaMemcpyAsync(m->in_ctc.get(), ctc_tgt, batch * S * 4, cudaMemcpyHostToDevice, st));
    TRBA_CHECK(cudaMemcpyAsync(m->in_ctc_len.get(), ctc_len, batch * 4, cudaMemcpyHostToDevice, st));
    int rc = trba_model_train_step(m, m->in_img.get(), m->in_text.get(), m->in_target.get(), m->in_ctc.get(),
                                   m->in_ctc_len.get(), batch, stream);
    if (rc) return rc;
    TRBA_CHECK(cudaMemcpyAsync(loss_host, m->loss.get(), 3 * sizeof(float), cudaMemcpyDeviceToHost, st));
    TRBA_CHECK(cudaStreamSynchronize(st));
    return cuda_status();
}

// Diagnostics: copy an internal fp32 buffer of the last step to the host.
// Names: feat, dfeat, enc, d_enc, logits, dlogits, ctc_logits, dctc,
// <conv>.x, <conv>.mean, <conv>.var; n must be the buffer's element count.
// Optimiser state and running statistics in and out (checkpoints).
int trba_model_get_moments(trba_model *m, float *m_host, float *v_host, long long n) {
    if (!m || n != m->n_params) return -1;
    if (m->cfg.inference_only) return training_refused(m);
    TRBA_CHECK(cudaDeviceSynchronize());
    if (m_host) TRBA_CHECK(cudaMemcpy(m_host, m->Mm.get(), n * 4, cudaMemcpyDeviceToHost));
    if (v_host) TRBA_CHECK(cudaMemcpy(v_host, m->Vv.get(), n * 4, cudaMemcpyDeviceToHost));
    return cuda_status();
}

int trba_model_set_moments(trba_model *m, const float *m_host, const float *v_host, long long n) {
    if (m && m->cfg.inference_only) return training_refused(m);
    if (!m || n != m->n_params) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    if (m_host) TRBA_CHECK(cudaMemcpy(m->Mm.get(), m_host, n * 4, cudaMemcpyHostToDevice));
    if (v_host) TRBA_CHECK(cudaMemcpy(m->Vv.get(), v_host, n * 4, cudaMemcpyHostToDevice));
    return cuda_status();
}

int trba_model_set_running_stats(trba_model *m, const float *host, long long n) {
    if (!m || !host || n != trba_model_running_stats_count(m)) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    long long o = 0;
    for (auto &L : m->convs) {
        TRBA_CHECK(cudaMemcpy(L.run_mean.get(), host + o, L.cout * 4, cudaMemcpyHostToDevice));
        TRBA_CHECK(cudaMemcpy(L.run_var.get(), host + o + L.cout, L.cout * 4, cudaMemcpyHostToDevice));
        o += 2 * L.cout;
    }
    return cuda_status();
}

int trba_model_set_step_count(trba_model *m, long long t) {
    if (!m || t < 0) return -1;
    TRBA_CHECK(cudaDeviceSynchronize());
    const double st[4] = {(double)t, 0.0, 0.0, 0.0};
    TRBA_CHECK(cudaMemcpy(m->step_state.get(), st, sizeof(st), cudaMemcpyHostToDevice));
    m->t = t;
    return cuda_status();
}

int trba_model_debug_tensor(trba_model *m, const char *name, float *host, long long n) {
    if (!m || !name || !host || n <= 0) return -1;
    const auto &cf = m->cfg;
    const i64 B = m->last_B, T = m->T, H = cf.hidden, V = cf.classes, S = m->steps;
    const std::string nm(name);
    const float *src = nullptr;
    i64 cnt = 0;
    if (nm == "feat") src = m->feat.get(), cnt = B * T * cf.fd;
    else if (nm == "dfeat") src = m->dfeat.get(), cnt = B * T * cf.fd;
    else if (nm == "enc") src = m->rnn.back().y.get(), cnt = B * T * H;
    else if (nm == "d_enc") src = m->d_bh.get(), cnt = B * T * H;
    else if (nm == "logits") src = m->logits.get(), cnt = S * B * V;
    else if (nm == "dlogits") src = m->dlogits.get(), cnt = S * B * V;
    else if (nm == "ctc_logits") src = m->ctc_logits.get(), cnt = B * T * V;
    else if (nm == "dctc") src = m->dctc.get(), cnt = B * T * V;
    else {
        for (auto &L : m->convs) {
            const i64 nx = B * L.cout * L.Ho * L.Wo;
            if (nm == L.name + ".x") src = L.x.get(), cnt = nx;
            else if (nm == L.name + ".mean") src = L.mean.get(), cnt = L.cout;
            else if (nm == L.name + ".var") src = L.var.get(), cnt = L.cout;
        }
    }
    if (!src || cnt != n) return -2;  // also: a training buffer of an inference-only model
    TRBA_CHECK(cudaDeviceSynchronize());
    TRBA_CHECK(cudaMemcpy(host, src, n * 4, cudaMemcpyDeviceToHost));
    return cuda_status();
}

int trba_model_probe(trba_model *m, int kind) {
    if (!m || kind < -1 || kind > TRBA_PROBE_PHASE_OPTIMIZER) return -1;
    if (m->gexec) {  // a recorded step graph may hold this probe's events
        TRBA_CHECK(cudaStreamSynchronize(m->gstream));
        TRBA_CHECK(cudaGraphExecDestroy(m->gexec));
        m->gexec = nullptr;
    }
    m->probe.kind = kind;
    m->probe.used = 0;
    m->probe.ops = 0.0;
    m->probe.bytes = 0.0;
    m->probe.steps = 0;
    m->probe.launches = 0;
    m->probe.nstamp = 0;
    m->probe.stamped = false;
    return 0;
}

int trba_model_probe_read(trba_model *m, double *ms_total, long long *launches, double *ops, double *bytes,
                          long long *steps) {
    if (!m || !ms_total || !launches || !ops || !bytes || !steps) return -1;
    auto &p = m->probe;
    double ms = 0.0;
    if (p.stamped) {  // launches of the latest replay of the step graph
        TRBA_CHECK(cudaStreamSynchronize(m->gstream));
        std::vector<unsigned long long> h(p.nstamp);
        TRBA_CHECK(cudaMemcpy(h.data(), p.stamps, p.nstamp * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i + 1 < p.nstamp; i += 2) ms += (double)(h[i + 1] - h[i]) * 1e-6;
    } else {
        if (p.used) TRBA_CHECK(cudaEventSynchronize(p.ev[p.used - 1]));
        for (size_t i = 0; i + 1 < p.used; i += 2) {
            float t = 0.0f;
            TRBA_CHECK(cudaEventElapsedTime(&t, p.ev[i], p.ev[i + 1]));
            ms += t;
        }
    }
    *ms_total = ms;
    *launches = p.launches;
    *ops = p.ops;
    *bytes = p.bytes;
    *steps = p.steps;
    return cuda_status();
}

int trba_dp_unique_id(void *id128) {
    if (!id128) return -1;
    if (!nccl().ok) {
        report_error(__FILE__, __LINE__, "libnccl.so.2 not found", -1);
        return -2;
    }
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return (int)r;
    std::memcpy(id128, &id, sizeof(id));
    return 0;
}

int trba_dp_init(trba_model *m, const void *id128, int rank, int world) {
    if (!m || !id128 || world < 1 || rank < 0 || rank >= world) return -1;
    if (m->cfg.inference_only) return training_refused(m);
    if (world == 1) return 0;
    if (!nccl().ok) {
        report_error(__FILE__, __LINE__, "libnccl.so.2 not found", -1);
        return -2;
    }
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    const ncclResult_t r = nccl().CommInitRank(&m->comm, world, id, rank);
    if (r != ncclSuccess) {
        report_error(__FILE__, __LINE__, nccl().GetErrorString(r), (int)r);
        m->comm = nullptr;
        return (int)r;
    }
    m->world = world;
    return 0;
}

// Watchdog over one step's completion (see include/trba_qat.h).
int trba_dp_watch(int (*stream_done)(void *), int (*async_error)(void *), void (*abort_comm)(void *), void *ctx,
                  double timeout_ms, double poll_us) {
    if (!stream_done || !async_error || !abort_comm) return -1;
    const auto t0 = std::chrono::steady_clock::now();
    const auto nap = std::chrono::microseconds((long long)(poll_us > 0 ? poll_us : 100.0));
    while (true) {
        const int d = stream_done(ctx);
        if (d < 0) return d;  // the stream reported an error of its own
        if (d > 0) return 0;
        const int e = async_error(ctx);
        if (e != 0) {
            abort_comm(ctx);
            return 1;
        }
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) {
            abort_comm(ctx);
            return 2;
        }
        std::this_thread::sleep_for(nap);
    }
}

int trba_dp_wait(trba_model *m, void *stream, double timeout_ms) {
    if (!m) return -1;
    struct Ctx {
        trba_model *m;
        cudaStream_t st;
    } c{m, as_stream(stream)};
    auto done = [](void *p) -> int {
        const cudaError_t e = cudaStreamQuery(static_cast<Ctx *>(p)->st);
        if (e == cudaSuccess) return 1;
        if (e == cudaErrorNotReady) return 0;
        return -(int)e;
    };
    auto async_err = [](void *p) -> int {
        trba_model *mm = static_cast<Ctx *>(p)->m;
        if (!mm->comm) return 0;
        ncclResult_t r = ncclSuccess;
        if (nccl().CommGetAsyncError(mm->comm, &r) != ncclSuccess) return -1;
        return r == ncclSuccess || r == ncclInProgress ? 0 : (int)r;
    };
    auto abort_comm = [](void *p) {
        trba_model *mm = static_cast<Ctx *>(p)->m;
        if (mm->comm) nccl().CommAbort(mm->comm);
        mm->comm = nullptr;
        mm->world = 1;
    };
    const int r = trba_dp_watch(done, async_err, abort_comm, &c, timeout_ms, 100.0);
    if (r == 1) report_error(__FILE__, __LINE__, "trba_dp_wait: NCCL reported an asynchronous error; aborted", -1);
    if (r == 2) report_error(__FILE__, __LINE__, "trba_dp_wait: step did not finish in time; NCCL aborted", -1);
    return r;
}

int trba_dp_finalize(trba_model *m) {
    if (!m) return -1;
    if (m->comm) {
        nccl().CommDestroy(m->comm);
        m->comm = nullptr;
    }
    m->world = 1;
    return 0;
}

}  // extern "C"
