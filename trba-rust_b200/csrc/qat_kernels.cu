// Fused element-wise / reduction kernels of the device-resident QAT step.
// Each kernel restates one or more of the reference's host-orchestrated
// launches (cited per kernel) with the same float expression order, written
// with explicit round-to-nearest intrinsics so that nothing is contracted.
#include <algorithm>

#include "qat_kernels.cuh"
#include "f32x2.cuh"

namespace trba {
namespace qat {
namespace {

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

// Block reductions (blockDim a multiple of 32, <= 1024).  Result in thread 0.
__device__ double block_sum_d(double v, double *sm) {
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sm[w] = v;
    __syncthreads();
    double r = 0.0;
    if (w == 0) {
        r = lane < nw ? sm[lane] : 0.0;
        r = warp_sum_d(r);
    }
    return r;
}
__device__ float block_max_f(float v, float *sm) {
    v = warp_max_f(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sm[w] = v;
    __syncthreads();
    float r = 0.0f;
    if (w == 0) {
        r = lane < nw ? sm[lane] : 0.0f;
        r = warp_max_f(r);
    }
    return r;
}

__device__ __forceinline__ void atomic_max_nonneg(float *p, float v) {
    atomicMax(reinterpret_cast<int *>(p), __float_as_int(v));
}

// BatchNorm statistics from the f64 sums (cpu_backend.cpp of the later
// snapshot, lines 762-767): mean = (float)s / cnt, var = max((float)q/cnt - m^2, 0).
__device__ __forceinline__ void bn_mean_var(const double *acc, int C, int c, i64 count, float &m, float &v) {
    const float cnt = (float)count;
    m = fdiv((float)acc[c], cnt);
    v = fsub(fdiv((float)acc[C + c], cnt), fmul(m, m));
    v = v < 0.0f ? 0.0f : v;
}
__device__ __forceinline__ float bn_rstd(float var) { return fdiv(1.0f, __fsqrt_rn(fadd(var, kBnEps))); }

// Per-plane view of a source: everything a thread needs for plane (b, c).
struct PlaneSrc {
    int kind;
    const float *x;
    float mean, r, gamma, beta, gate, res_s;
    const float *res_f;
    const int8_t *res_q;
    __device__ __forceinline__ float one(float xv, i64 i) const {
        switch (kind) {
            case SRC_BN: return fadd(fmul(fmul(fsub(xv, mean), r), gamma), beta);
            case SRC_FLOAT: return xv;
            case SRC_SE_RES_F: return fadd(fmul(xv, gate), res_f[i]);
            default: return fadd(fmul(xv, gate), fmul((float)res_q[i], res_s));
        }
    }
    __device__ __forceinline__ float at(i64 i) const { return one(x[i], i); }
    // Four consecutive elements from a 16-byte aligned index i.
    __device__ __forceinline__ float4 at4(i64 i) const {
        const float4 xv = *reinterpret_cast<const float4 *>(x + i);
        float4 v;
        switch (kind) {
            case SRC_BN:
                v.x = fadd(fmul(fmul(fsub(xv.x, mean), r), gamma), beta);
                v.y = fadd(fmul(fmul(fsub(xv.y, mean), r), gamma), beta);
                v.z = fadd(fmul(fmul(fsub(xv.z, mean), r), gamma), beta);
                v.w = fadd(fmul(fmul(fsub(xv.w, mean), r), gamma), beta);
                return v;
            case SRC_FLOAT: return xv;
            case SRC_SE_RES_F: {
                const float4 rf = *reinterpret_cast<const float4 *>(res_f + i);
                v.x = fadd(fmul(xv.x, gate), rf.x);
                v.y = fadd(fmul(xv.y, gate), rf.y);
                v.z = fadd(fmul(xv.z, gate), rf.z);
                v.w = fadd(fmul(xv.w, gate), rf.w);
                return v;
            }
            default: {
                const char4 rq = *reinterpret_cast<const char4 *>(res_q + i);
                v.x = fadd(fmul(xv.x, gate), fmul((float)rq.x, res_s));
                v.y = fadd(fmul(xv.y, gate), fmul((float)rq.y, res_s));
                v.z = fadd(fmul(xv.z, gate), fmul((float)rq.z, res_s));
                v.w = fadd(fmul(xv.w, gate), fmul((float)rq.w, res_s));
                return v;
            }
        }
    }
};

// Planes whose length is a multiple of 4 are read as float4 (all buffers
// are 256-byte aligned, so a plane starting at a multiple of 4 elements is
// 16-byte aligned).
__device__ __forceinline__ bool vec4_ok(int HW) { return (HW & 3) == 0; }

// Planes of HW elements are processed one per warp when small (8 planes per
// 256-thread CTA) and one per CTA otherwise; PlaneIdx says which plane a
// thread works on, its index inside the plane's thread group and the group's
// width.  Reductions over a plane are warp shuffles or a block reduction.
constexpr int kWarpPlaneMaxHW = 1024;

struct PlaneIdx {
    int plane, lane, width;
    bool live, leader;
};

__device__ __forceinline__ PlaneIdx plane_idx(int nplanes, int warp_mode) {
    PlaneIdx q;
    if (warp_mode) {
        q.plane = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        q.lane = threadIdx.x & 31;
        q.width = 32;
    } else {
        q.plane = blockIdx.x;
        q.lane = threadIdx.x;
        q.width = blockDim.x;
    }
    q.live = q.plane < nplanes;
    if (!q.live) q.plane = nplanes - 1;  // valid reads; no writes
    q.leader = q.live && q.lane == 0;
    return q;
}

// Sum over a plane's thread group; valid in the group's lane 0.
__device__ __forceinline__ double plane_sum_d(double v, int warp_mode, double *sm) {
    return warp_mode ? warp_sum_d(v) : block_sum_d(v, sm);
}

__device__ PlaneSrc plane_src(const Src &s, int b, int c, bool leader, float *mean_out = nullptr,
                              float *var_out = nullptr) {
    PlaneSrc p;
    p.kind = s.kind;
    p.x = s.x;
    p.mean = p.r = p.gamma = p.beta = p.gate = p.res_s = 0.0f;
    p.res_f = s.res_f;
    p.res_q = s.res_q;
    if (s.kind == SRC_BN_EVAL) {  // src/qnet.rs:871-876: mean / var are the running statistics
        p.kind = SRC_BN;
        p.mean = s.run_mean[c];
        p.r = bn_rstd(s.run_var[c]);
        p.gamma = s.gamma[c];
        p.beta = s.beta[c];
    } else if (s.kind == SRC_BN) {
        float m, v;
        bn_mean_var(s.bn_acc, s.C, c, s.count, m, v);
        p.mean = m;
        p.r = bn_rstd(v);
        p.gamma = s.gamma[c];
        p.beta = s.beta[c];
        if (mean_out && b == 0 && leader) {
            mean_out[c] = m;
            var_out[c] = v;
        }
    } else if (s.kind == SRC_SE_RES_F || s.kind == SRC_SE_RES_Q) {
        p.gate = s.gate[(i64)b * s.C + c];
        if (s.kind == SRC_SE_RES_Q) p.res_s = *s.res_s;
    }
    return p;
}

// ------------------------------------------------------------- forward --
// src/qnet.rs:877-895 (bn_apply), 1212-1214 (avgpool_hw of y2),
// 1102-1106 (reduce_max_abs before relu_quant).
__global__ void act_stats_kernel(Src s, int nplanes, int warp_mode, float *y_out, float *mean_out, float *var_out,
                                 float *pool_out, float *vmax) {
    __shared__ double smd[32];
    __shared__ float smf[32];
    const PlaneIdx q = plane_idx(nplanes, warp_mode);
    const int b = q.plane / s.C, c = q.plane - b * s.C;
    const PlaneSrc p = plane_src(s, b, c, q.leader, mean_out, var_out);
    const i64 base = (i64)q.plane * s.HW;
    double sum = 0.0;
    float mx = 0.0f;
    if (q.live) {
        if (vec4_ok(s.HW)) {
            for (int j = 4 * q.lane; j < s.HW; j += 4 * q.width) {
                const float4 v = p.at4(base + j);
                if (y_out) *reinterpret_cast<float4 *>(y_out + base + j) = v;
                sum += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
        } else {
            for (int j = q.lane; j < s.HW; j += q.width) {
                const float v = p.at(base + j);
                if (y_out) y_out[base + j] = v;
                sum += (double)v;
                mx = fmaxf(mx, fabsf(v));
            }
        }
    }
    if (pool_out) {
        const double t = plane_sum_d(sum, warp_mode, smd);
        if (q.leader) pool_out[q.plane] = (float)(t / (double)s.HW);
    }
    if (vmax) {
        const float m = block_max_f(mx, smf);
        if (threadIdx.x == 0) atomic_max_nonneg(vmax, m);
    }
}

__global__ void act_quant_kernel(Src s, int nplanes, int warp_mode, const float *vmax, float *s_out, int8_t *qo,
                                 int relu) {
    const PlaneIdx q = plane_idx(nplanes, warp_mode);
    if (!q.live) return;
    const int b = q.plane / s.C, c = q.plane - b * s.C;
    const PlaneSrc p = plane_src(s, b, c, q.leader);
    const float sc = fmaxf(fdiv(*vmax, 127.0f), 1e-12f);
    const float inv = fdiv(1.0f, sc);
    if (q.plane == 0 && q.leader && s_out) *s_out = sc;
    const i64 base = (i64)q.plane * s.HW;
    auto quant = [&](float v) -> int8_t {
        const float t = relu ? fminf(fmul(fmaxf(v, 0.0f), inv), 127.0f) : fminf(fmaxf(fmul(v, inv), -127.0f), 127.0f);
        return (int8_t)rint_even(t);
    };
    if (vec4_ok(s.HW)) {
        for (int j = 4 * q.lane; j < s.HW; j += 4 * q.width) {
            const float4 v = p.at4(base + j);
            *reinterpret_cast<char4 *>(qo + base + j) = make_char4(quant(v.x), quant(v.y), quant(v.z), quant(v.w));
        }
    } else {
        for (int j = q.lane; j < s.HW; j += q.width) qo[base + j] = quant(p.at(base + j));
    }
}

int plane_threads(int HW) { return HW >= 256 ? 256 : HW > 64 ? 128 : HW > 32 ? 64 : 32; }

// src/qnet.rs:1219-1222: pre1 = fc1 pool, h1 = relu, pre2 = fc2 h1, gate = sigmoid.
__global__ void se_forward_kernel(const float *pool, const float *w1, const float *w2, int C, int R, float *h1,
                                  float *gate) {
    extern __shared__ float sm[];
    float *sp = sm, *sh = sm + C;
    const int b = blockIdx.x;
    for (int i = threadIdx.x; i < C; i += blockDim.x) sp[i] = pool[(i64)b * C + i];
    __syncthreads();
    for (int j = threadIdx.x; j < R; j += blockDim.x) {
        double acc = 0.0;
        for (int i = 0; i < C; ++i) acc = fma((double)sp[i], (double)w1[(i64)j * C + i], acc);
        const float h = fmaxf((float)acc, 0.0f);
        sh[j] = h;
        h1[(i64)b * R + j] = h;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        double acc = 0.0;
        for (int j = 0; j < R; ++j) acc = fma((double)sh[j], (double)w2[(i64)c * R + j], acc);
        gate[(i64)b * C + c] = cr_sigmoid((float)acc);
    }
}

// ------------------------------------------------------------ backward --
// Block-gradient entry and SE backward in one pass over each sample
// (src/qnet.rs:1684-1708, 1290-1296 and 1298-1330).  One CTA per sample:
//   dz = q_out > 0 ? rint(clamp(gv * s_out / s_dq)) * s_dq : 0, written out
//     (the residual and downsample gradients read it later), with
//     s_dq = max(vmax / 127, 1e-12), vmax = max |gv * s_out| over the batch
//     (accumulated by the gather that wrote gv);
//   the squeeze sum over each plane of dz * y2 (f64), one warp per plane,
//     kSeRows planes' reductions overlapped, kSeCols positions per lane
//     loaded ahead;
//   the excitation MLP backward (one warp per hidden unit, then one thread
//     per channel) and dy2_full = dz * gate + dpooled / HW.
constexpr int kSeRows = 4;
constexpr int kSeCols = 2;

__global__ void __launch_bounds__(256, 4) se_backward_kernel(
    const float *__restrict__ gv, const float *__restrict__ s_out, const float *__restrict__ vmax,
    const int8_t *__restrict__ q_out, float *__restrict__ s_dq_out, float *dz,
    const float *__restrict__ y2, const float *__restrict__ gate, const float *__restrict__ h1,
    const float *__restrict__ w1, const float *__restrict__ w2, int C, int HW, int R, float *__restrict__ dpre1,
    float *__restrict__ dpre2, float *__restrict__ dpooled, float *__restrict__ dy2_full) {
    extern __shared__ float sm[];
    float *s_dp2 = sm, *s_dp1 = sm + C, *s_gate = sm + C + R, *s_add = s_gate + C;
    const int b = blockIdx.x;
    const i64 base = (i64)b * C * HW;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const float s = *s_out;
    const float sdq = fmaxf(fdiv(*vmax, 127.0f), 1e-12f);
    const float inv = fdiv(1.0f, sdq);
    if (b == 0 && threadIdx.x == 0 && s_dq_out) *s_dq_out = sdq;
    for (int c0 = warp; c0 < C; c0 += nwarps * kSeRows) {
        double acc[kSeRows];
#pragma unroll
        for (int u = 0; u < kSeRows; ++u) acc[u] = 0.0;
        // kSeRows planes x kSeCols positions per lane per pass: every load of
        // the pass is issued before the first use, so the planes' loads are in
        // flight together; each lane still adds its positions j = lane,
        // lane + 32, ... in increasing order (the f64 sums are unchanged).
        for (int j0 = lane; j0 < HW; j0 += 32 * kSeCols) {
            float gvv[kSeRows][kSeCols], y2v[kSeRows][kSeCols];
            int8_t qv[kSeRows][kSeCols];
#pragma unroll
            for (int u = 0; u < kSeRows; ++u)
#pragma unroll
                for (int t = 0; t < kSeCols; ++t) {
                    const int c = c0 + u * nwarps, j = j0 + 32 * t;
                    const bool ok = c < C && j < HW;
                    const i64 e = base + (i64)c * HW + j;
                    gvv[u][t] = ok ? gv[e] : 0.0f;
                    y2v[u][t] = ok ? y2[e] : 0.0f;
                    qv[u][t] = ok ? q_out[e] : (int8_t)0;
                }
#pragma unroll
            for (int u = 0; u < kSeRows; ++u)
#pragma unroll
                for (int t = 0; t < kSeCols; ++t) {
                    const int c = c0 + u * nwarps, j = j0 + 32 * t;
                    if (c < C && j < HW) {
                        const float v = fmul(gvv[u][t], s);
                        const int qd = rint_even(fminf(fmaxf(fmul(v, inv), -127.0f), 127.0f));
                        const float d = qv[u][t] > 0 ? fmul((float)qd, sdq) : 0.0f;
                        dz[base + (i64)c * HW + j] = d;
                        acc[u] += (double)fmul(d, y2v[u][t]);
                    }
                }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int u = 0; u < kSeRows; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
        if (lane == 0) {
#pragma unroll
            for (int u = 0; u < kSeRows; ++u) {
                const int c = c0 + u * nwarps;
                if (c >= C) break;
                const float pm = (float)(acc[u] / (double)HW);
                const float dgate = fmul(pm, (float)HW);
                const float g = gate[(i64)b * C + c];
                const float d2 = fmul(fmul(dgate, g), fsub(1.0f, g));
                s_dp2[c] = d2;
                s_gate[c] = g;
                dpre2[(i64)b * C + c] = d2;
            }
        }
    }
    __syncthreads();
    for (int j = warp; j < R; j += nwarps) {
        double acc = 0.0;
        for (int c = lane; c < C; c += 32) acc = fma((double)s_dp2[c], (double)w2[(i64)c * R + j], acc);
        acc = warp_sum_d(acc);
        if (lane == 0) {
            const float d1 = h1[(i64)b * R + j] > 0.0f ? (float)acc : 0.0f;
            s_dp1[j] = d1;
            dpre1[(i64)b * R + j] = d1;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        double acc = 0.0;
        for (int j = 0; j < R; ++j) acc = fma((double)s_dp1[j], (double)w1[(i64)j * C + i], acc);
        const float dp = (float)acc;
        dpooled[(i64)b * C + i] = dp;
        s_add[i] = fdiv(dp, (float)HW);
    }
    __syncthreads();
    if ((HW & 3) == 0) {
        // four float4 per thread per pass, loaded before any is stored (dz and
        // dy2_full are distinct buffers)
        const int hw4 = HW >> 2, n4 = C * hw4;
        const float4 *z4 = reinterpret_cast<const float4 *>(dz + base);
        float4 *o4 = reinterpret_cast<float4 *>(dy2_full + base);
        for (int e0 = threadIdx.x; e0 < n4; e0 += 4 * blockDim.x) {
            float4 z[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int e = e0 + t * blockDim.x;
                z[t] = e < n4 ? z4[e] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int e = e0 + t * blockDim.x;
                if (e < n4) {
                    const int c = e / hw4;
                    const float g = s_gate[c], ad = s_add[c];
                    o4[e] = make_float4(fadd(fmul(z[t].x, g), ad), fadd(fmul(z[t].y, g), ad),
                                        fadd(fmul(z[t].z, g), ad), fadd(fmul(z[t].w, g), ad));
                }
            }
        }
    } else {
        for (int e = threadIdx.x; e < C * HW; e += blockDim.x) {
            const int c = e / HW;
            dy2_full[base + e] = fadd(fmul(dz[base + e], s_gate[c]), s_add[c]);
        }
    }
}

// g_w2[c, j] += sum_b dpre2[b,c] h1[b,j];  g_w1[j, i] += sum_b dpre1[b,j] pool[b,i]
// One warp per weight: lanes stride over the batch, f64 products summed
// with a warp reduction and rounded once.
__global__ void se_wgrad_kernel(const float *dpre1, const float *dpre2, const float *h1, const float *pool, int B,
                                int C, int R, float *g_w1, float *g_w2) {
    const int n2 = C * R;
    const i64 e = (i64)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (e >= 2 * (i64)n2) return;
    double acc = 0.0;
    if (e < n2) {
        const int c = (int)(e / R), j = (int)(e - (i64)c * R);
        for (int b = lane; b < B; b += 32) acc = fma((double)dpre2[(i64)b * C + c], (double)h1[(i64)b * R + j], acc);
        acc = warp_sum_d(acc);
        if (lane == 0) g_w2[e] = fadd(g_w2[e], (float)acc);
    } else {
        const i64 f = e - n2;
        const int j = (int)(f / C), i = (int)(f - (i64)j * C);
        for (int b = lane; b < B; b += 32)
            acc = fma((double)dpre1[(i64)b * R + j], (double)pool[(i64)b * C + i], acc);
        acc = warp_sum_d(acc);
        if (lane == 0) g_w1[f] = fadd(g_w1[f], (float)acc);
    }
}

// Warp-per-channel-group form of the per-plane BN backward passes (planes
// of at most kWarpPlaneMaxHW elements): a warp takes the planes of channel c
// of images b0 .. b0 + G - 1 (G = bn_group(HW)), walks their elements as one
// list with kBnAhead loads of dy and x per lane in flight, and reduces once
// for the whole group (one shuffle tree and one pair of atomics per G planes
// instead of per plane).
constexpr int kBnAhead = 4;
__host__ __device__ inline int bn_group(int HW) {
    const int g = (640 + HW - 1) / HW;
    return g < 1 ? 1 : (g > 16 ? 16 : g);
}
struct BnGroup {
    int c, b0, n;  // channel, first image, images in the group (0: idle warp)
};
__device__ __forceinline__ BnGroup bn_group_of(int B, int C, int G) {
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int per_c = (B + G - 1) / G;
    BnGroup g;
    g.c = gw % C;
    g.b0 = (gw / C) * G;
    g.n = gw < C * per_c ? min(G, B - g.b0) : 0;
    return g;
}
// f(dy, x) over the group's elements, kBnAhead float4 (or scalars when HW is
// not a multiple of 4) per lane loaded before any is used.
template <typename F>
__device__ __forceinline__ void bn_group_walk(const float *dy, const float *x, int C, int HW, const BnGroup &g,
                                              int lane, F &&f) {
    if (vec4_ok(HW)) {
        const int n4 = HW >> 2, total = g.n * n4;
        for (int e0 = lane; e0 < total; e0 += 32 * kBnAhead) {
            float4 d[kBnAhead], xv[kBnAhead];
#pragma unroll
            for (int u = 0; u < kBnAhead; ++u) {
                const int e = e0 + 32 * u;
                if (e < total) {
                    const int gi = e / n4, j4 = e - gi * n4;
                    const i64 i = ((i64)(g.b0 + gi) * C + g.c) * HW + 4 * j4;
                    d[u] = *reinterpret_cast<const float4 *>(dy + i);
                    xv[u] = *reinterpret_cast<const float4 *>(x + i);
                }
            }
#pragma unroll
            for (int u = 0; u < kBnAhead; ++u)
                if (e0 + 32 * u < total) {
                    f(d[u].x, xv[u].x);
                    f(d[u].y, xv[u].y);
                    f(d[u].z, xv[u].z);
                    f(d[u].w, xv[u].w);
                }
        }
    } else {
        const int total = g.n * HW;
        for (int e0 = lane; e0 < total; e0 += 32 * kBnAhead) {
            float d[kBnAhead], xv[kBnAhead];
#pragma unroll
            for (int u = 0; u < kBnAhead; ++u) {
                const int e = e0 + 32 * u;
                if (e < total) {
                    const int gi = e / HW, j = e - gi * HW;
                    const i64 i = ((i64)(g.b0 + gi) * C + g.c) * HW + j;
                    d[u] = dy[i];
                    xv[u] = x[i];
                }
            }
#pragma unroll
            for (int u = 0; u < kBnAhead; ++u)
                if (e0 + 32 * u < total) f(d[u], xv[u]);
        }
    }
}

// later snapshot cpu_backend.cpp:782-802, one CTA per (b, c) plane, f64
// partials added into acc[c] (sum dy) and acc[C + c] (sum dy*xhat).
__global__ void bn_bwd_sums_kernel(const float *dy, const float *x, const float *mean, const float *var, int C,
                                   int HW, int nplanes, int warp_mode, double *acc) {
    __shared__ double smd[32];
    if (warp_mode) {
        const BnGroup g = bn_group_of(nplanes / C, C, bn_group(HW));
        if (g.n == 0) return;
        const float m = mean[g.c], r = bn_rstd(var[g.c]);
        double s = 0.0, sx = 0.0;
        bn_group_walk(dy, x, C, HW, g, threadIdx.x & 31, [&](float d, float xv) {
            s += (double)d;
            sx += (double)fmul(d, fmul(fsub(xv, m), r));
        });
        s = warp_sum_d(s);
        sx = warp_sum_d(sx);
        if ((threadIdx.x & 31) == 0) {
            atomicAdd(acc + g.c, s);
            atomicAdd(acc + C + g.c, sx);
        }
        return;
    }
    const PlaneIdx q = plane_idx(nplanes, warp_mode);
    const int c = q.plane % C;
    const float m = mean[c], r = bn_rstd(var[c]);
    const i64 base = (i64)q.plane * HW;
    double s = 0.0, sx = 0.0;
    if (q.live) {
        if (vec4_ok(HW)) {
            for (int j = 4 * q.lane; j < HW; j += 4 * q.width) {
                const float4 d = *reinterpret_cast<const float4 *>(dy + base + j);
                const float4 xv = *reinterpret_cast<const float4 *>(x + base + j);
                s += (double)d.x + (double)d.y + (double)d.z + (double)d.w;
                sx += (double)fmul(d.x, fmul(fsub(xv.x, m), r)) + (double)fmul(d.y, fmul(fsub(xv.y, m), r)) +
                      (double)fmul(d.z, fmul(fsub(xv.z, m), r)) + (double)fmul(d.w, fmul(fsub(xv.w, m), r));
            }
        } else {
            for (int j = q.lane; j < HW; j += q.width) {
                const float d = dy[base + j];
                const float xh = fmul(fsub(x[base + j], m), r);
                s += (double)d;
                sx += (double)fmul(d, xh);
            }
        }
    }
    const double ts = plane_sum_d(s, warp_mode, smd);
    const double tx = plane_sum_d(sx, warp_mode, smd);
    if (q.leader) {
        atomicAdd(acc + c, ts);
        atomicAdd(acc + C + c, tx);
    }
}

struct DxPlane {
    float m, r, a, sdy, sdxh, cnt;
};
__device__ DxPlane dx_plane(const float *mean, const float *var, const float *gamma, const double *acc, int C, int c,
                            i64 count) {
    DxPlane p;
    p.m = mean[c];
    p.r = bn_rstd(var[c]);
    p.cnt = (float)count;
    p.a = fdiv(fmul(gamma[c], p.r), p.cnt);
    p.sdy = (float)acc[c];
    p.sdxh = (float)acc[C + c];
    return p;
}
// later snapshot cpu_backend.cpp:804-817
__device__ __forceinline__ float dx_at(const DxPlane &p, float dy, float x) {
    const float xh = fmul(fsub(x, p.m), p.r);
    return fmul(p.a, fsub(fsub(fmul(p.cnt, dy), p.sdy), fmul(xh, p.sdxh)));
}

__global__ void bn_dx_max_kernel(const float *dy, const float *x, const float *mean, const float *var,
                                 const float *gamma, const double *acc, int B, int C, int HW, int nplanes,
                                 int warp_mode, float *g_gamma, float *g_beta, float *vmax) {
    __shared__ float smf[32];
    if (warp_mode) {
        const BnGroup g = bn_group_of(B, C, bn_group(HW));
        float mx = 0.0f;
        if (g.n > 0) {
            const DxPlane p = dx_plane(mean, var, gamma, acc, C, g.c, (i64)B * HW);
            if (g.b0 == 0 && (threadIdx.x & 31) == 0) {  // src/qnet.rs:974-982
                g_beta[g.c] = fadd(g_beta[g.c], p.sdy);
                g_gamma[g.c] = fadd(g_gamma[g.c], p.sdxh);
            }
            bn_group_walk(dy, x, C, HW, g, threadIdx.x & 31,
                          [&](float d, float xv) { mx = fmaxf(mx, fabsf(dx_at(p, d, xv))); });
        }
        const float t = block_max_f(mx, smf);
        if (threadIdx.x == 0) atomic_max_nonneg(vmax, t);
        return;
    }
    const PlaneIdx q = plane_idx(nplanes, warp_mode);
    const int b = q.plane / C, c = q.plane - b * C;
    const DxPlane p = dx_plane(mean, var, gamma, acc, C, c, (i64)B * HW);
    if (b == 0 && q.leader) {  // src/qnet.rs:974-982: g_beta += sum dy, g_gamma += sum dy xhat
        g_beta[c] = fadd(g_beta[c], p.sdy);
        g_gamma[c] = fadd(g_gamma[c], p.sdxh);
    }
    const i64 base = (i64)q.plane * HW;
    float mx = 0.0f;
    if (q.live) {
        if (vec4_ok(HW)) {
            for (int j = 4 * q.lane; j < HW; j += 4 * q.width) {
                const float4 d = *reinterpret_cast<const float4 *>(dy + base + j);
                const float4 xv = *reinterpret_cast<const float4 *>(x + base + j);
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(dx_at(p, d.x, xv.x)), fabsf(dx_at(p, d.y, xv.y))),
                                     fmaxf(fabsf(dx_at(p, d.z, xv.z)), fabsf(dx_at(p, d.w, xv.w)))));
            }
        } else {
            for (int j = q.lane; j < HW; j += q.width) mx = fmaxf(mx, fabsf(dx_at(p, dy[base + j], x[base + j])));
        }
    }
    const float t = block_max_f(mx, smf);
    if (threadIdx.x == 0) atomic_max_nonneg(vmax, t);
}

__device__ __forceinline__ int8_t quant_dx(float d, float inv) {
    return (int8_t)rint_even(fminf(fmaxf(fmul(d, inv), -127.0f), 127.0f));
}

// dx quantised into the wgrad operand laid out [C, rows] (dW = dX^T col):
// A[c * ld + b*HW + j].
__global__ void bn_dx_quant_kernel(const float *dy, const float *x, const float *mean, const float *var,
                                   const float *gamma, const double *acc, int B, int C, int HW, int nplanes,
                                   int warp_mode, const float *vmax, float *s_dx, int8_t *A, int ld) {
    const PlaneIdx q = plane_idx(nplanes, warp_mode);
    if (!q.live) return;
    const int b = q.plane / C, c = q.plane - b * C;
    const DxPlane p = dx_plane(mean, var, gamma, acc, C, c, (i64)B * HW);
    const float sc = fmaxf(fdiv(*vmax, 127.0f), 1e-12f);
    const float inv = fdiv(1.0f, sc);
    if (q.plane == 0 && q.leader) *s_dx = sc;
    const i64 base = (i64)q.plane * HW;
    int8_t *arow = A + (i64)c * ld + (i64)b * HW;
    if (vec4_ok(HW)) {
        for (int j = 4 * q.lane; j < HW; j += 4 * q.width) {
            const float4 d = *reinterpret_cast<const float4 *>(dy + base + j);
            const float4 xv = *reinterpret_cast<const float4 *>(x + base + j);
            *reinterpret_cast<char4 *>(arow + j) =
                make_char4(quant_dx(dx_at(p, d.x, xv.x), inv), quant_dx(dx_at(p, d.y, xv.y), inv),
                           quant_dx(dx_at(p, d.z, xv.z), inv), quant_dx(dx_at(p, d.w, xv.w), inv));
        }
    } else {
        for (int j = q.lane; j < HW; j += q.width) arow[j] = quant_dx(dx_at(p, dy[base + j], x[base + j]), inv);
    }
}

// The reference-compatible operand (src/qnet.rs:984-1001: transpose_i8 of the
// NCHW dx buffer viewed as [rows, C]): A[o * ld + r] = q(dx_flat[r * C + o]).
// 32 x 32 tiles through shared memory: the reads walk dx_flat contiguously,
// the writes walk A's rows contiguously.  Per-channel BN terms for all C
// channels sit in shared memory.
constexpr int kQtTile = 32;

// Division of 32-bit unsigned numerators by a run-time constant d >= 1:
// n / d = umulhi(n, m) >> s with m, s chosen on the host (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994;
// the round-up method with a 33-bit multiplier, split as 2^32 + m).
struct FastDiv {
    uint32_t d, m, s;
    __host__ static FastDiv make(uint32_t d) {
        FastDiv f;
        f.d = d;
        uint32_t l = 0;
        while ((1ull << l) < d) ++l;  // l = ceil(log2 d)
        f.m = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
        f.s = l;
        return f;
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        const uint32_t t = __umulhi(n, m);
        return s == 0 ? n : (t + ((n - t) >> 1)) >> (s - 1);
    }
};

__global__ void __launch_bounds__(256) bn_dx_quant_t_kernel(const float *dy, const float *x, const float *mean,
                                                            const float *var, const float *gamma,
                                                            const double *acc, int B, int C, int HW,
                                                            const float *vmax, float *s_dx, int8_t *A, int ld,
                                                            i64 rows, FastDiv div_hw, FastDiv div_c) {
    extern __shared__ float chs[];  // [5][C]: m, r, a, sdy, sdxh
    __shared__ int8_t tile[kQtTile][kQtTile + 4];
    const i64 count = (i64)B * HW;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const DxPlane p = dx_plane(mean, var, gamma, acc, C, c, count);
        chs[c] = p.m;
        chs[C + c] = p.r;
        chs[2 * C + c] = p.a;
        chs[3 * C + c] = p.sdy;
        chs[4 * C + c] = p.sdxh;
    }
    __syncthreads();
    const float sc = fmaxf(fdiv(*vmax, 127.0f), 1e-12f);
    const float inv = fdiv(1.0f, sc);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *s_dx = sc;
    const float cnt = (float)count;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const i64 r0 = (i64)blockIdx.x * kQtTile;
    const int o0 = blockIdx.y * kQtTile;
    for (int k = ty; k < kQtTile; k += blockDim.x >> 5) {
        const i64 r = r0 + k;
        const int o = o0 + tx;
        int8_t v = 0;
        if (r < rows && o < C) {
            const i64 i = r * C + o;
            const uint32_t plane = div_hw.div((uint32_t)i);
            const int c = (int)(plane - div_c.div(plane) * (uint32_t)C);
            DxPlane p;
            p.m = chs[c];
            p.r = chs[C + c];
            p.a = chs[2 * C + c];
            p.sdy = chs[3 * C + c];
            p.sdxh = chs[4 * C + c];
            p.cnt = cnt;
            v = quant_dx(dx_at(p, dy[i], x[i]), inv);
        }
        tile[tx][k] = v;
    }
    __syncthreads();
    for (int k = ty; k < kQtTile; k += blockDim.x >> 5) {
        const int o = o0 + k;
        const i64 r = r0 + tx;
        if (o < C && r < rows) A[(i64)o * ld + r] = tile[k][tx];
    }
}

// Small-C form of the same operand (C % 4 == 0, HW % 4 == 0, C <= 512): a
// CTA takes R whole rows of the [rows, C] view, R = (8192 / C) rounded down
// to 16.  Thread (o, rows 4j..4j+3) quantises four elements of column o (a
// coalesced read across the warp's consecutive columns) into one 32-bit word
// of a [C][R + 4] byte tile; each of the C operand rows then receives its R
// bytes as 16-byte stores.  With C = 16 or 32 the 32 x 32 tiles above leave
// half their threads idle and write 32-byte row pieces.
constexpr int kQtElems = 8192;
__host__ __device__ inline int qt_rows(int C) { return (kQtElems / C) & ~15; }

__global__ void __launch_bounds__(256) bn_dx_quant_tr_kernel(const float *dy, const float *x, const float *mean,
                                                             const float *var, const float *gamma,
                                                             const double *acc, int B, int C, int HW,
                                                             const float *vmax, float *s_dx, int8_t *A, int ld,
                                                             i64 rows, FastDiv div_hw, FastDiv div_c) {
    extern __shared__ float chs[];  // [5][C]: m, r, a, sdy, sdxh
    __shared__ __align__(16) uint32_t tile[(kQtElems + 4 * 512) / 4];  // [C][R + 4] bytes
    const i64 count = (i64)B * HW;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const DxPlane p = dx_plane(mean, var, gamma, acc, C, c, count);
        chs[c] = p.m;
        chs[C + c] = p.r;
        chs[2 * C + c] = p.a;
        chs[3 * C + c] = p.sdy;
        chs[4 * C + c] = p.sdxh;
    }
    __syncthreads();
    const float sc = fmaxf(fdiv(*vmax, 127.0f), 1e-12f);
    const float inv = fdiv(1.0f, sc);
    if (blockIdx.x == 0 && threadIdx.x == 0) *s_dx = sc;
    const float cnt = (float)count;
    const int R = qt_rows(C), RW = R / 4 + 1;  // tile row stride in words
    const i64 r0 = (i64)blockIdx.x * R;
    const int nrows = (int)min((i64)R, rows - r0);
    const int quads = (nrows + 3) >> 2;
    // two quads (eight rows) of one column per thread per pass: the sixteen
    // loads of dy and x are issued before any is used
    for (int k0 = threadIdx.x; k0 < C * quads; k0 += 2 * blockDim.x) {
        float dv[2][4], xv[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int k = k0 + h * blockDim.x;
            const int q4 = k / C, o = k - q4 * C;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = 4 * q4 + j;
                const bool ok = k < C * quads && r < nrows;
                const uint32_t i = ok ? (uint32_t)((r0 + r) * C + o) : 0u;
                dv[h][j] = ok ? dy[i] : 0.0f;
                xv[h][j] = ok ? x[i] : 0.0f;
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int k = k0 + h * blockDim.x;
            if (k >= C * quads) break;
            const int q4 = k / C, o = k - q4 * C;
            uint32_t word = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = 4 * q4 + j;
                if (r < nrows) {
                    const uint32_t i = (uint32_t)((r0 + r) * C + o);
                    const uint32_t plane = div_hw.div(i);
                    const int c = (int)(plane - div_c.div(plane) * (uint32_t)C);
                    DxPlane p;
                    p.m = chs[c];
                    p.r = chs[C + c];
                    p.a = chs[2 * C + c];
                    p.sdy = chs[3 * C + c];
                    p.sdxh = chs[4 * C + c];
                    p.cnt = cnt;
                    word |= (uint32_t)(uint8_t)quant_dx(dx_at(p, dv[h][j], xv[h][j]), inv) << (8 * j);
                }
            }
            tile[o * RW + q4] = word;
        }
    }
    __syncthreads();
    if (nrows == R) {
        const int cpr = R / 16;  // 16-byte pieces per operand row
        for (int k = threadIdx.x; k < C * cpr; k += blockDim.x) {
            const int o = k / cpr, j = k - o * cpr;
            const uint32_t *t = tile + o * RW + 4 * j;
            *reinterpret_cast<int4 *>(A + (i64)o * ld + r0 + 16 * j) =
                make_int4((int)t[0], (int)t[1], (int)t[2], (int)t[3]);
        }
    } else {
        const int8_t *tb = reinterpret_cast<const int8_t *>(tile);
        for (int k = threadIdx.x; k < C * nrows; k += blockDim.x) {
            const int o = k / nrows, j = k - o * nrows;
            A[(i64)o * ld + r0 + j] = tb[4 * o * RW + j];
        }
    }
}

__global__ void grad_accum_kernel(const int32_t *acc, const float *s_dx, const float *s_in, i64 n, float *g) {
    const float deq = fmul(*s_dx, *s_in);
    GRID_LOOP(i, n) g[i] = fadd(g[i], fmul((float)acc[i], deq));
}

// Input gradient (src/qnet.rs:1068-1080 -> launch_conv_backward_grad_input_i8).
//
// Every output gi[b, ci, ih, iw] is accumulated in the reference's order —
// taps (kh, kw) outer, output channels inner, one f32 multiply and one f32
// add per term, both rounded — then scaled by w_s, so the result is
// bit-identical to the reference's per-element gather.
//
// A thread owns one input pixel x 16 input channels (8 packed accumulator
// pairs).  The CTA's weights, (float) of the int8 weights laid out
// [tap][oc][16 channels] by the re-quantisation (dgrad_weights_index), are
// copied into shared memory once and read as 64-bit pairs broadcast to the
// whole warp; each dy value loaded feeds 16 accumulators.  The arithmetic runs
// on the packed f32x2 pipe (prod2_rn / add2_rn: separately rounded multiply
// and add).  A tap outside the output plane is skipped, exactly as the
// reference skips it.
//
// Pixel order: with `perm` null thread t takes pixel t (row-major over
// images).  Otherwise pixels are grouped into classes (`perm` lists the
// image-local pixels class by class, `cstart` the class offsets), class-major
// over the batch, so the lanes of a warp share their taps and no lane idles
// on a tap that only its neighbours need.  Strided convs group by the full set
// of valid taps (in the natural order half or more of the lanes would idle);
// stride-1 convs group by the valid kernel rows only, which keeps each warp
// on contiguous row segments of dy (grouping by columns as well breaks rows
// into short runs and measured slower on 4 x 20 planes).
constexpr int kDgradCi = 16, kDgradThreads = 256;

__global__ void __launch_bounds__(kDgradThreads, 3) dgrad_kernel(
    const float *__restrict__ go, const float *__restrict__ wT, const float *__restrict__ w_s, int B, int Cin, int H,
    int W, int Cout, int kH, int kW, int sH, int sW, int pH, int pW, int Ho, int Wo, const int *__restrict__ perm,
    const int *__restrict__ cstart, int ncls, const int8_t *__restrict__ mask_q, const float *__restrict__ add,
    float *__restrict__ gi, float neg_zero, const float *__restrict__ gmax_scale, float *__restrict__ gmax_out) {
    constexpr int CI = kDgradCi, NP = CI / 2;
    extern __shared__ float4 wsm4[];  // [taps][Cout][CI / 4]
    const int khw = kH * kW, ci0 = blockIdx.y * CI;
    {
        const float4 *src = reinterpret_cast<const float4 *>(wT) + (i64)blockIdx.y * khw * Cout * (CI / 4);
        for (int e = threadIdx.x; e < khw * Cout * (CI / 4); e += kDgradThreads) wsm4[e] = src[e];
    }
    __syncthreads();
    const int hwo = Ho * Wo, hwi = H * W;
    const i64 t = (i64)blockIdx.x * kDgradThreads + threadIdx.x;
    // threads past the end take part in the optional max reduction only
    const bool live = t < (i64)B * hwi;
    float gmax = 0.0f;
    if (live) {
        int b, pix;
        if (perm) {
            int c = 0;
            while (c + 1 < ncls && t >= (i64)B * cstart[c + 1]) ++c;
            const int c0 = cstart[c], csz = cstart[c + 1] - c0;
            const i64 local = t - (i64)B * c0;
            b = (int)(local / csz);
            pix = perm[c0 + (int)(local - (i64)b * csz)];
        } else {
            b = (int)(t / hwi);
            pix = (int)(t - (i64)b * hwi);
        }
        const int ih = pix / W, iw = pix - ih * W;
        const f32x2 z = pack2(neg_zero, neg_zero);
        f32x2 acc[NP];
#pragma unroll
        for (int j = 0; j < NP; ++j) acc[j] = 0ull;  // (+0, +0)
        const float *gob = go + (i64)b * Cout * hwo;
        for (int kh = 0; kh < kH; ++kh) {
            const int nh = ih + pH - kh;
            if (nh < 0 || nh % sH != 0 || nh / sH >= Ho) continue;
            for (int kw = 0; kw < kW; ++kw) {
                const int nw = iw + pW - kw;
                if (nw < 0 || nw % sW != 0 || nw / sW >= Wo) continue;
                const float *gp = gob + (nh / sH) * Wo + nw / sW;
                const ulonglong2 *wt = reinterpret_cast<const ulonglong2 *>(wsm4) + (i64)(kh * kW + kw) * Cout * (CI / 4);
#pragma unroll 8
                for (int oc = 0; oc < Cout; ++oc) {
                    f32x2 wv[NP];
#pragma unroll
                    for (int q = 0; q < CI / 4; ++q) {
                        const ulonglong2 w2 = wt[(CI / 4) * oc + q];
                        wv[2 * q] = w2.x;
                        wv[2 * q + 1] = w2.y;
                    }
                    const float d = gp[(i64)oc * hwo];
                    const f32x2 dd = pack2(d, d);
#pragma unroll
                    for (int j = 0; j < NP; ++j) acc[j] = add2_rn(acc[j], prod2_rn(dd, wv[j], z));
                }
            }
        }
        const float ws = *w_s;
        float a[CI];
#pragma unroll
        for (int j = 0; j < NP; ++j) unpack2(acc[j], a[2 * j], a[2 * j + 1]);
#pragma unroll
        for (int j = 0; j < CI; ++j) {
            const int ci = ci0 + j;
            if (ci >= Cin) break;
            const i64 i = ((i64)b * Cin + ci) * hwi + pix;
            float v = fmul(a[j], ws);
            if (mask_q) v = mask_q[i] > 0 ? v : 0.0f;
            if (add) v = fadd(v, add[i]);
            gi[i] = v;
            if (gmax_out) gmax = fmaxf(gmax, fabsf(fmul(v, *gmax_scale)));
        }
    }
    if (gmax_out) {
        // max |gi * gmax_scale| over the launch (the next block's
        // re-quantisation scale): one atomic per CTA
        __shared__ float wmax[kDgradThreads / 32];
        const float m = block_max_f(gmax, wmax);
        if (threadIdx.x == 0) atomic_max_nonneg(gmax_out, m);
    }
}

__global__ void im2col_t_kernel(const int8_t *in, int8_t *colT, int C, int H, int W, int kH, int kW, int sH, int sW,
                                int pH, int pW, int Ho, int Wo, i64 rows, int ld) {
    const int cols = C * kH * kW, khw = kH * kW;
    GRID_LOOP(e, (i64)cols * rows) {
        const int n = (int)(e / rows);
        const i64 r = e - (i64)n * rows;
        const i64 b = r / ((i64)Ho * Wo);
        const int rem = (int)(r - b * Ho * Wo), oh = rem / Wo, ow = rem - oh * Wo;
        const int ci = n / khw, kk = n - ci * khw, kh = kk / kW, kw = kk - kh * kW;
        const int ih = oh * sH + kh - pH, iw = ow * sW + kw - pW;
        int8_t v = 0;
        if (ih >= 0 && ih < H && iw >= 0 && iw < W) v = in[((b * C + ci) * H + ih) * W + iw];
        colT[(i64)n * ld + r] = v;
    }
}

__global__ void pool_bwd_mask_kernel(const int8_t *q1, const float *gv, const float *s_pool, int H, int W, i64 n,
                                     float *dy) {
    const float sp = *s_pool;
    const int Ho = H >> 1, Wo = W >> 1;
    GRID_LOOP(i, n) {
        const i64 bc = i / ((i64)H * W);
        const int pix = (int)(i - bc * H * W), ih = pix / W, iw = pix - ih * W;
        const int oh = ih >> 1, ow = iw >> 1;
        const i64 wb = bc * H * W + (i64)(2 * oh) * W + 2 * ow;
        const int8_t *w = q1 + wb;
        int win = 0;
        int8_t m = w[0];
        if (w[1] > m) { m = w[1]; win = 1; }
        if (w[W] > m) { m = w[W]; win = W; }
        if (w[W + 1] > m) { m = w[W + 1]; win = W + 1; }
        float v = 0.0f;
        if (wb + win == i) v = fmul(gv[bc * Ho * Wo + (i64)oh * Wo + ow], sp);
        dy[i] = q1[i] > 0 ? v : 0.0f;
    }
}

// Fast path of pool_bwd_mask for H even and W % 4 == 0: one thread per two
// horizontally adjacent 2x2 windows (4-byte q1 loads, 16-byte dy stores,
// 32-bit index arithmetic within a plane).  Same first-maximum rule.
__device__ __forceinline__ void pool_win_bwd(int8_t a, int8_t b, int8_t c, int8_t d, float g, float &oa, float &ob,
                                             float &oc, float &od) {
    int win = 0;
    int8_t m = a;
    if (b > m) { m = b; win = 1; }
    if (c > m) { m = c; win = 2; }
    if (d > m) win = 3;
    oa = (win == 0 && a > 0) ? g : 0.0f;
    ob = (win == 1 && b > 0) ? g : 0.0f;
    oc = (win == 2 && c > 0) ? g : 0.0f;
    od = (win == 3 && d > 0) ? g : 0.0f;
}

__global__ void pool_bwd_mask4_kernel(const int8_t *__restrict__ q1, const float *__restrict__ gv,
                                      const float *__restrict__ s_pool, int H, int W, int BC, float *__restrict__ dy) {
    const float sp = *s_pool;
    const int Ho = H >> 1, Wo = W >> 1, W4 = W >> 2, per = Ho * W4;
    for (int bc = blockIdx.y; bc < BC; bc += gridDim.y) {
        const int8_t *qp = q1 + (i64)bc * H * W;
        const float *gp = gv + (i64)bc * Ho * Wo;
        float *dp = dy + (i64)bc * H * W;
        for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < per; k += gridDim.x * blockDim.x) {
            const int oh = k / W4, q = k - oh * W4;
            const int o = 2 * oh * W + 4 * q;
            const char4 r0 = *reinterpret_cast<const char4 *>(qp + o);
            const char4 r1 = *reinterpret_cast<const char4 *>(qp + o + W);
            const float2 g = *reinterpret_cast<const float2 *>(gp + oh * Wo + 2 * q);
            float4 t, u;
            pool_win_bwd(r0.x, r0.y, r1.x, r1.y, fmul(g.x, sp), t.x, t.y, u.x, u.y);
            pool_win_bwd(r0.z, r0.w, r1.z, r1.w, fmul(g.y, sp), t.z, t.w, u.z, u.w);
            *reinterpret_cast<float4 *>(dp + o) = t;
            *reinterpret_cast<float4 *>(dp + o + W) = u;
        }
    }
}

__global__ void features_kernel(const int8_t *q, const float *s, int C, int H, int W, i64 total, float *feat) {
    const float sc = *s;
    GRID_LOOP(i, total) {
        const int c = (int)(i % C), w = (int)((i / C) % W);
        const i64 b = i / ((i64)C * W);
        const int8_t *p = q + ((b * C + c) * H) * W + w;
        float acc = 0.0f;
        for (int h = 0; h < H; ++h) acc = fadd(acc, fmul((float)p[(i64)h * W], sc));
        feat[i] = fdiv(acc, (float)H);
    }
}

__global__ void features_bwd_kernel(const float *dfeat, const int8_t *q, const float *s, int C, int H, int W,
                                    i64 n, float *dy) {
    const float sc = *s;
    GRID_LOOP(i, n) {
        const i64 bc = i / ((i64)H * W);
        const int pix = (int)(i - bc * H * W), w = pix % W;
        const i64 b = bc / C;
        const int c = (int)(bc - b * C);
        const float v = fmul(fdiv(dfeat[(b * W + w) * C + c], (float)H), sc);
        dy[i] = q[i] > 0 ? v : 0.0f;
    }
}

__global__ void mask_by_q_kernel(const int8_t *q, const float *g, i64 n, float *dy) {
    GRID_LOOP(i, n) dy[i] = q[i] > 0 ? g[i] : 0.0f;
}

}  // namespace

struct PlaneLaunch {
    int grid, threads, warp_mode;
};
PlaneLaunch plane_launch(i64 nplanes, int HW) {
    if (HW <= kWarpPlaneMaxHW) return {(int)((nplanes + 7) / 8), 256, 1};
    return {(int)nplanes, plane_threads(HW), 0};
}

void act_stats(const Src &s, int B, float *y_out, float *mean_out, float *var_out, float *pool_out, float *vmax,
               cudaStream_t st) {
    const int np = B * s.C;
    const PlaneLaunch L = plane_launch(np, s.HW);
    act_stats_kernel<<<L.grid, L.threads, 0, st>>>(s, np, L.warp_mode, y_out, mean_out, var_out, pool_out, vmax);
    TRBA_LAUNCH_CHECK();
}

void act_quant(const Src &s, int B, const float *vmax, float *s_out, int8_t *q, bool relu, cudaStream_t st) {
    const int np = B * s.C;
    const PlaneLaunch L = plane_launch(np, s.HW);
    act_quant_kernel<<<L.grid, L.threads, 0, st>>>(s, np, L.warp_mode, vmax, s_out, q, relu ? 1 : 0);
    TRBA_LAUNCH_CHECK();
}

void se_forward(const float *pool, const float *w1, const float *w2, int B, int C, int R, float *h1, float *gate,
                cudaStream_t st) {
    se_forward_kernel<<<B, 128, (C + R) * sizeof(float), st>>>(pool, w1, w2, C, R, h1, gate);
    TRBA_LAUNCH_CHECK();
}

void se_backward(const float *gv, const float *s_out, const float *vmax, const int8_t *q_out, float *s_dq_out,
                 float *dz, const float *y2, const float *gate, const float *h1, const float *w1, const float *w2,
                 int B, int C, int HW, int R, float *dpre1, float *dpre2, float *dpooled, float *dy2_full,
                 cudaStream_t st) {
    TRBA_REQUIRE((i64)C * HW < (1ll << 31), "se_backward: sample plane set too large for 32-bit indexing");
    se_backward_kernel<<<B, 256, (3 * C + R) * sizeof(float), st>>>(gv, s_out, vmax, q_out, s_dq_out, dz, y2, gate,
                                                                   h1, w1, w2, C, HW, R, dpre1, dpre2, dpooled,
                                                                   dy2_full);
    TRBA_LAUNCH_CHECK();
}

void se_weight_grads(const float *dpre1, const float *dpre2, const float *h1, const float *pool, int B, int C, int R,
                     float *g_w1, float *g_w2, cudaStream_t st) {
    const i64 warps = 2LL * C * R;
    se_wgrad_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(dpre1, dpre2, h1, pool, B, C, R, g_w1, g_w2);
    TRBA_LAUNCH_CHECK();
}

// Grid of the BN backward passes: warp mode launches one warp per (channel,
// group of bn_group(HW) images).
PlaneLaunch bn_launch(int B, int C, int HW) {
    PlaneLaunch L = plane_launch((i64)B * C, HW);
    if (L.warp_mode) {
        const i64 warps = (i64)C * ((B + bn_group(HW) - 1) / bn_group(HW));
        L.grid = (int)((warps + 7) / 8);
    }
    return L;
}

void bn_bwd_sums(const float *dy, const float *x, const float *mean, const float *var, int B, int C, int HW,
                 double *acc, cudaStream_t st) {
    const int np = B * C;
    const PlaneLaunch L = bn_launch(B, C, HW);
    bn_bwd_sums_kernel<<<L.grid, L.threads, 0, st>>>(dy, x, mean, var, C, HW, np, L.warp_mode, acc);
    TRBA_LAUNCH_CHECK();
}

void bn_dx_max(const float *dy, const float *x, const float *mean, const float *var, const float *gamma,
               const double *acc, int B, int C, int HW, float *g_gamma, float *g_beta, float *vmax, cudaStream_t st) {
    const int np = B * C;
    const PlaneLaunch L = bn_launch(B, C, HW);
    bn_dx_max_kernel<<<L.grid, L.threads, 0, st>>>(dy, x, mean, var, gamma, acc, B, C, HW, np, L.warp_mode, g_gamma,
                                                   g_beta, vmax);
    TRBA_LAUNCH_CHECK();
}

void bn_dx_quant(const float *dy, const float *x, const float *mean, const float *var, const float *gamma,
                 const double *acc, int B, int C, int HW, const float *vmax, float *s_dx, int8_t *A, int ld,
                 bool compat, cudaStream_t st) {
    if (compat) {
        const i64 rows = (i64)B * HW;
        TRBA_REQUIRE(rows * C < (1ll << 32), "bn_dx_quant: tensor too large for 32-bit indexing");
        if (C % 4 == 0 && C <= 512 && HW % 4 == 0 && ld % 16 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0) {
            const int R = qt_rows(C);
            bn_dx_quant_tr_kernel<<<(unsigned)((rows + R - 1) / R), 256, 5 * C * sizeof(float), st>>>(
                dy, x, mean, var, gamma, acc, B, C, HW, vmax, s_dx, A, ld, rows, FastDiv::make(HW), FastDiv::make(C));
            TRBA_LAUNCH_CHECK();
            return;
        }
        dim3 grid((unsigned)((rows + kQtTile - 1) / kQtTile), (unsigned)((C + kQtTile - 1) / kQtTile));
        bn_dx_quant_t_kernel<<<grid, 256, 5 * C * sizeof(float), st>>>(dy, x, mean, var, gamma, acc, B, C, HW, vmax,
                                                                        s_dx, A, ld, rows, FastDiv::make(HW),
                                                                        FastDiv::make(C));
    } else {
        const int np = B * C;
        const PlaneLaunch L = plane_launch(np, HW);
        bn_dx_quant_kernel<<<L.grid, L.threads, 0, st>>>(dy, x, mean, var, gamma, acc, B, C, HW, np, L.warp_mode,
                                                         vmax, s_dx, A, ld);
    }
    TRBA_LAUNCH_CHECK();
}

void grad_accum(const int32_t *acc, const float *s_dx, const float *s_in, i64 n, float *g, cudaStream_t st) {
    grad_accum_kernel<<<grid_for(n), 256, 0, st>>>(acc, s_dx, s_in, n, g);
    TRBA_LAUNCH_CHECK();
}

i64 dgrad_weights_size(int Cin, int Cout, int khw) { return (i64)((Cin + kDgradCi - 1) / kDgradCi) * khw * Cout * kDgradCi; }

void dgrad_classes(int H, int W, int kh, int kw, int sh, int sw, int ph, int pw, int Ho, int Wo, bool rows_only,
                   std::vector<int> &perm, std::vector<int> &cstart) {
    std::vector<std::pair<unsigned long long, int>> key;
    key.reserve((size_t)H * W);
    for (int ih = 0; ih < H; ++ih)
        for (int iw = 0; iw < W; ++iw) {
            unsigned long long m = 0;
            for (int a = 0; a < kh; ++a)
                for (int c = 0; c < kw; ++c) {
                    const int nh = ih + ph - a, nw = iw + pw - c;
                    const bool row_ok = nh >= 0 && nh % sh == 0 && nh / sh < Ho;
                    if (rows_only ? row_ok : row_ok && nw >= 0 && nw % sw == 0 && nw / sw < Wo)
                        m |= 1ull << ((a * kw + c) & 63);
                }
            key.push_back({m, ih * W + iw});
        }
    std::stable_sort(key.begin(), key.end(), [](const std::pair<unsigned long long, int> &x,
                                                const std::pair<unsigned long long, int> &y) { return x.first > y.first; });
    perm.clear();
    cstart.clear();
    for (size_t i = 0; i < key.size(); ++i) {
        if (i == 0 || key[i].first != key[i - 1].first) cstart.push_back((int)i);
        perm.push_back(key[i].second);
    }
    cstart.push_back((int)key.size());
    if (cstart.size() <= 2) {  // one class: the natural order
        perm.clear();
        cstart.clear();
    }
}

void dgrad(const float *dy, const float *wT, const float *w_s, int B, int Cin, int H, int W, int Cout, int kh, int kw,
           int sh, int sw, int ph, int pw, int Ho, int Wo, const int *perm, const int *cstart, int ncls,
           const int8_t *mask_q, const float *add, float *gi, cudaStream_t st, const float *gmax_scale,
           float *gmax_out) {
    const i64 npix = (i64)B * H * W;
    if (npix <= 0 || Cin <= 0) return;
    const size_t smem = sizeof(float) * (size_t)kh * kw * Cout * kDgradCi;
    TRBA_REQUIRE(smem <= 200 * 1024, "dgrad: kernel taps x output channels too large for shared memory");
    TRBA_REQUIRE(kh * kw <= 64, "dgrad: at most 64 kernel taps");
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && dev >= 0 && dev < 64 && !attr[dev]) {
        TRBA_CHECK(cudaFuncSetAttribute(dgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr[dev] = true;
    }
    dim3 grid((unsigned)((npix + kDgradThreads - 1) / kDgradThreads), (unsigned)((Cin + kDgradCi - 1) / kDgradCi));
    dgrad_kernel<<<grid, kDgradThreads, smem, st>>>(dy, wT, w_s, B, Cin, H, W, Cout, kh, kw, sh, sw, ph, pw, Ho, Wo,
                                                    perm, cstart, perm ? ncls : 0, mask_q, add, gi, -0.0f,
                                                    gmax_out ? gmax_scale : nullptr, gmax_scale ? gmax_out : nullptr);
    TRBA_LAUNCH_CHECK();
}

void im2col_t(const int8_t *in, int8_t *colT, int B, int C, int H, int W, int kh, int kw, int sh, int sw, int ph,
              int pw, int Ho, int Wo, int ld, cudaStream_t st) {
    const i64 rows = (i64)B * Ho * Wo;
    im2col_t_kernel<<<grid_for((i64)C * kh * kw * rows), 256, 0, st>>>(in, colT, C, H, W, kh, kw, sh, sw, ph, pw, Ho,
                                                                       Wo, rows, ld);
    TRBA_LAUNCH_CHECK();
}

void pool_bwd_mask(const int8_t *q1, const float *gv, const float *s_pool, int B, int C, int H, int W, float *dy,
                   cudaStream_t st) {
    const i64 n = (i64)B * C * H * W;
    if ((H & 1) == 0 && (W & 3) == 0 && (i64)H * W < (1ll << 30)) {
        const int BC = B * C, per = (H >> 1) * (W >> 2);
        dim3 grid((unsigned)((per + 255) / 256), (unsigned)(BC < 65535 ? BC : 65535));
        pool_bwd_mask4_kernel<<<grid, 256, 0, st>>>(q1, gv, s_pool, H, W, BC, dy);
    } else {
        pool_bwd_mask_kernel<<<grid_for(n), 256, 0, st>>>(q1, gv, s_pool, H, W, n, dy);
    }
    TRBA_LAUNCH_CHECK();
}

void features(const int8_t *q, const float *s, int B, int C, int H, int W, float *feat, cudaStream_t st) {
    const i64 total = (i64)B * W * C;
    features_kernel<<<grid_for(total), 256, 0, st>>>(q, s, C, H, W, total, feat);
    TRBA_LAUNCH_CHECK();
}

void features_bwd(const float *dfeat, const int8_t *q, const float *s, int B, int C, int H, int W, float *dy,
                  cudaStream_t st) {
    const i64 n = (i64)B * C * H * W;
    features_bwd_kernel<<<grid_for(n), 256, 0, st>>>(dfeat, q, s, C, H, W, n, dy);
    TRBA_LAUNCH_CHECK();
}

void mask_by_q(const int8_t *q, const float *g, i64 n, float *dy, cudaStream_t st) {
    mask_by_q_kernel<<<grid_for(n), 256, 0, st>>>(q, g, n, dy);
    TRBA_LAUNCH_CHECK();
}

}  // namespace qat
}  // namespace trba
