// fp32 BiLSTM time-slot kernels of the drop-in ABI (reference later snapshot
// src/backend.rs:70-90, device path src/rnn.rs:504-841).  Layouts: x/dx
// [B, T, D]; gates/dgates [T, B, 4H] (post-activation, PyTorch order
// i, f, g, o); c/h traces [T, B, H] in slot order (slot s of the reverse
// direction is time position T-1-s).
#include "common.cuh"

namespace {

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per (b, i): four gate dot products over D (+H), then the cell.
__global__ void lstm_fwd_step_kernel(const float *__restrict__ x, const float *__restrict__ w_ih,
                                     const float *__restrict__ b_ih, const float *__restrict__ w_hh,
                                     const float *__restrict__ b_hh, float *__restrict__ gates,
                                     float *__restrict__ c_out, float *__restrict__ h_out, i64 B,
                                     i64 T, i64 D, i64 H, i64 slot, i64 tt) {
    const i64 warp = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= B * H) return;
    const i64 bi = warp / H, i = warp - bi * H;
    const float *xr = x + (bi * T + tt) * D;
    const float *hp = slot ? h_out + ((slot - 1) * B + bi) * H : nullptr;
    float g[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const i64 o = q * H + i;
        float s = 0.0f;
        for (i64 k = lane; k < D; k += 32) s += xr[k] * w_ih[o * D + k];
        if (hp)
            for (i64 k = lane; k < H; k += 32) s += hp[k] * w_hh[o * H + k];
        g[q] = warp_sum(s) + (b_ih[o] + b_hh[o]);
    }
    if (lane == 0) {
        const float ig = sigmoidf_(g[0]), fg = sigmoidf_(g[1]), cg = tanhf(g[2]), og = sigmoidf_(g[3]);
        const float cp = slot ? c_out[((slot - 1) * B + bi) * H + i] : 0.0f;
        const float cn = fg * cp + ig * cg;
        const i64 gs = (slot * B + bi) * 4 * H, cs = (slot * B + bi) * H;
        gates[gs + i] = ig;
        gates[gs + H + i] = fg;
        gates[gs + 2 * H + i] = cg;
        gates[gs + 3 * H + i] = og;
        c_out[cs + i] = cn;
        h_out[cs + i] = og * tanhf(cn);
    }
}

__global__ void lstm_bwd_cell_kernel(const float *__restrict__ dh_out, const float *__restrict__ gates,
                                     const float *__restrict__ ctrace, const float *__restrict__ dh_next,
                                     const float *__restrict__ dc_next, float *__restrict__ dgates,
                                     float *__restrict__ dc_next_out, i64 B, i64 H, i64 slot) {
    GRID_LOOP(idx, B * H) {
        const i64 bi = idx / H, i = idx - bi * H;
        const i64 cs = (slot * B + bi) * H, gs = (slot * B + bi) * 4 * H;
        const float cp = slot ? ctrace[((slot - 1) * B + bi) * H + i] : 0.0f;
        const float ig = gates[gs + i], fg = gates[gs + H + i], cg = gates[gs + 2 * H + i],
                    og = gates[gs + 3 * H + i];
        const float tc = tanhf(ctrace[cs + i]);
        const float dh = dh_out[cs + i] + dh_next[bi * H + i];
        const float dc = dh * og * (1.0f - tc * tc) + dc_next[bi * H + i] * fg;
        dgates[gs + i] = dc * cg * ig * (1.0f - ig);
        dgates[gs + H + i] = dc * cp * fg * (1.0f - fg);
        dgates[gs + 2 * H + i] = dc * ig * (1.0f - cg * cg);
        dgates[gs + 3 * H + i] = dh * tc * og * (1.0f - og);
        dc_next_out[bi * H + i] = dc;
    }
}

// One thread per (b, k), k < D writes dx[b, tt, k], k >= D writes dh_next.
__global__ void lstm_bwd_rec_kernel(const float *__restrict__ dgates, const float *__restrict__ w_ih,
                                    const float *__restrict__ w_hh, float *__restrict__ dx,
                                    float *__restrict__ dh_next, i64 B, i64 T, i64 D, i64 H, i64 slot,
                                    i64 tt) {
    GRID_LOOP(idx, B * (D + H)) {
        const i64 bi = idx / (D + H), k = idx - bi * (D + H);
        const float *dg = dgates + (slot * B + bi) * 4 * H;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        if (k < D) {
            i64 o = 0;
            for (; o + 3 < 4 * H; o += 4) {
                s0 += dg[o] * w_ih[o * D + k];
                s1 += dg[o + 1] * w_ih[(o + 1) * D + k];
                s2 += dg[o + 2] * w_ih[(o + 2) * D + k];
                s3 += dg[o + 3] * w_ih[(o + 3) * D + k];
            }
            for (; o < 4 * H; ++o) s0 += dg[o] * w_ih[o * D + k];
            dx[(bi * T + tt) * D + k] = (s0 + s1) + (s2 + s3);
        } else {
            const i64 kk = k - D;
            i64 o = 0;
            for (; o + 3 < 4 * H; o += 4) {
                s0 += dg[o] * w_hh[o * H + kk];
                s1 += dg[o + 1] * w_hh[(o + 1) * H + kk];
                s2 += dg[o + 2] * w_hh[(o + 2) * H + kk];
                s3 += dg[o + 3] * w_hh[(o + 3) * H + kk];
            }
            for (; o < 4 * H; ++o) s0 += dg[o] * w_hh[o * H + kk];
            dh_next[bi * H + kk] = (s0 + s1) + (s2 + s3);
        }
    }
}

__global__ void lstm_wgrad_ih_kernel(const float *__restrict__ dgates, const float *__restrict__ x,
                                     float *__restrict__ g_w, i64 B, i64 T, i64 D, i64 H, int rev,
                                     int accumulate) {
    GRID_LOOP(idx, 4 * H * D) {
        const i64 o = idx / D, k = idx - o * D;
        float s = 0.0f;
        for (i64 j = 0; j < T * B; ++j) {
            const i64 slot = j / B, bi = j - slot * B, tt = rev ? T - 1 - slot : slot;
            s += dgates[j * 4 * H + o] * x[(bi * T + tt) * D + k];
        }
        g_w[idx] = accumulate ? g_w[idx] + s : s;
    }
}

__global__ void lstm_wgrad_hh_kernel(const float *__restrict__ dgates, const float *__restrict__ htrace,
                                     float *__restrict__ g_w, i64 B, i64 T, i64 H, int accumulate) {
    GRID_LOOP(idx, 4 * H * H) {
        const i64 o = idx / H, k = idx - o * H;
        float s = 0.0f;
        for (i64 j = B; j < T * B; ++j) {
            const i64 slot = j / B, bi = j - slot * B;
            s += dgates[j * 4 * H + o] * htrace[((slot - 1) * B + bi) * H + k];
        }
        g_w[idx] = accumulate ? g_w[idx] + s : s;
    }
}

__global__ void lstm_bgrad_kernel(const float *__restrict__ dgates, float *__restrict__ g_b_ih,
                                  float *__restrict__ g_b_hh, i64 B, i64 T, i64 H, int accumulate) {
    GRID_LOOP(o, 4 * H) {
        float s = 0.0f;
        for (i64 j = 0; j < T * B; ++j) s += dgates[j * 4 * H + o];
        g_b_ih[o] = accumulate ? g_b_ih[o] + s : s;
        g_b_hh[o] = accumulate ? g_b_hh[o] + s : s;
    }
}

}  // namespace

using namespace trba;

extern "C" {

void launch_lstm_fwd_step(const float *x, const float *w_ih, const float *b_ih, const float *w_hh,
                          const float *b_hh, float *gates, float *c_out, float *h_out, i64 B, i64 T,
                          i64 D, i64 H, i64 slot, i64 rev, void *s) {
    if (B <= 0 || T <= 0 || D <= 0 || H <= 0 || slot < 0 || slot >= T) return;
    const i64 threads = B * H * 32;
    const int grid = (int)((threads + 255) / 256);
    lstm_fwd_step_kernel<<<grid, 256, 0, as_stream(s)>>>(x, w_ih, b_ih, w_hh, b_hh, gates, c_out, h_out,
                                                         B, T, D, H, slot, rev ? T - 1 - slot : slot);
    TRBA_LAUNCH_CHECK();
}

void launch_lstm_bwd_cell(const float *dh_out, const float *gates, const float *ctrace,
                          const float *dh_next, const float *dc_next, float *dgates,
                          float *dc_next_out, i64 B, i64 H, i64 slot, void *s) {
    if (B <= 0 || H <= 0) return;
    lstm_bwd_cell_kernel<<<grid_for(B * H), 256, 0, as_stream(s)>>>(dh_out, gates, ctrace, dh_next,
                                                                    dc_next, dgates, dc_next_out, B, H,
                                                                    slot);
    TRBA_LAUNCH_CHECK();
}

void launch_lstm_bwd_rec(const float *dgates, const float *w_ih, const float *w_hh, float *dx,
                         float *dh_next, i64 B, i64 T, i64 D, i64 H, i64 slot, i64 rev, void *s) {
    if (B <= 0 || T <= 0 || D <= 0 || H <= 0) return;
    lstm_bwd_rec_kernel<<<grid_for(B * (D + H)), 256, 0, as_stream(s)>>>(
        dgates, w_ih, w_hh, dx, dh_next, B, T, D, H, slot, rev ? T - 1 - slot : slot);
    TRBA_LAUNCH_CHECK();
}

void launch_lstm_wgrad_ih(const float *dgates, const float *x, float *g_w, i64 B, i64 T, i64 D, i64 H,
                          i64 rev, i64 accumulate, void *s) {
    if (B <= 0 || T <= 0 || D <= 0 || H <= 0) return;
    lstm_wgrad_ih_kernel<<<grid_for(4 * H * D), 256, 0, as_stream(s)>>>(dgates, x, g_w, B, T, D, H,
                                                                        rev ? 1 : 0, accumulate ? 1 : 0);
    TRBA_LAUNCH_CHECK();
}

void launch_lstm_wgrad_hh(const float *dgates, const float *htrace, float *g_w, i64 B, i64 T, i64 H,
                          i64 accumulate, void *s) {
    if (B <= 0 || T <= 0 || H <= 0) return;
    lstm_wgrad_hh_kernel<<<grid_for(4 * H * H), 256, 0, as_stream(s)>>>(dgates, htrace, g_w, B, T, H,
                                                                        accumulate ? 1 : 0);
    TRBA_LAUNCH_CHECK();
}

void launch_lstm_bgrad(const float *dgates, float *g_b_ih, float *g_b_hh, i64 B, i64 T, i64 H,
                       i64 accumulate, void *s) {
    if (B <= 0 || T <= 0 || H <= 0) return;
    lstm_bgrad_kernel<<<grid_for(4 * H), 256, 0, as_stream(s)>>>(dgates, g_b_ih, g_b_hh, B, T, H,
                                                                 accumulate ? 1 : 0);
    TRBA_LAUNCH_CHECK();
}

}  // extern "C"
