"""Table of seeded calls covering every compute entry point of the backend
ABI (include/trba_backend.h), runnable through any backend adapter of
tests/kat_runner.py.  Each case names the function, its arguments (input
arrays, output arrays with a poison fill, or scalars) and how its outputs are
compared: bit-exact, or within a stated tolerance.

Sizes are chosen to cover ragged tails (not multiples of 16, 32 or 128),
stride-2 and 1x1 convolutions and the conv_out 2x2 s(2,1) p(0,1) geometry of
the reference network, while keeping the CPU oracle under a second per case.
"""
from __future__ import annotations

import numpy as np

from kat import a16


class In:
    def __init__(self, a):
        self.a = np.ascontiguousarray(a)


class Out:
    def __init__(self, shape, dtype, fill=0, tol="exact"):
        self.shape, self.dtype, self.fill, self.tol = shape, dtype, fill, tol


def _rng(seed):
    return np.random.default_rng(seed)


def _i8(rng, n, lo=-127, hi=128):
    return rng.integers(lo, hi, size=n, dtype=np.int64).astype(np.int8)


def _f32(rng, n, s=1.0):
    return (rng.standard_normal(n) * s).astype(np.float32)


def conv_geoms():
    # (b, cin, h, w, cout, kh, kw, sh, sw, ph, pw)
    return [
        (2, 3, 9, 11, 5, 3, 3, 1, 1, 1, 1),
        (3, 6, 8, 10, 7, 3, 3, 2, 2, 1, 1),
        (2, 5, 7, 7, 9, 1, 1, 2, 2, 0, 0),
        (2, 8, 4, 9, 8, 2, 2, 2, 1, 0, 1),   # conv_out.0 geometry
        (1, 8, 2, 10, 8, 2, 2, 1, 1, 0, 0),  # conv_out.3 geometry
        (2, 16, 6, 13, 4, 3, 3, 1, 1, 1, 1),  # stem.3 channel count (row-per-thread im2col)
        (2, 3, 7, 9, 4, 3, 3, 2, 2, 1, 1),    # 3 channels, strided
        (2, 16, 5, 12, 4, 3, 3, 1, 1, 1, 1),  # stem.3 form, W % 4 == 0 (four-pixel im2col)
        (3, 3, 4, 8, 5, 3, 3, 1, 1, 1, 1),    # stem.0 form, W % 4 == 0
        (2, 32, 5, 9, 8, 3, 3, 1, 1, 1, 1),   # C % 16 == 0: row-segment im2col
        (2, 64, 6, 7, 16, 3, 3, 2, 2, 1, 1),  # the same, strided
        (1, 32, 4, 9, 8, 2, 2, 2, 1, 0, 1),   # the same, conv_out.0 geometry
        (2, 48, 5, 6, 8, 1, 1, 2, 2, 0, 0),   # the same, 1x1 stride 2
    ]


def out_hw(g):
    b, cin, h, w, cout, kh, kw, sh, sw, ph, pw = g
    return (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1


def cases():
    """Yields (case_id, function_name, [args])."""
    R = _rng(20261201)
    # ---- GEMMs
    for (m, n, k) in [(1, 1, 1), (33, 17, 5), (129, 40, 200), (300, 96, 144), (257, 300, 130)]:
        kp = a16(k)
        A = np.zeros((a16(m), kp), np.int8)
        B = np.zeros((a16(n), kp), np.int8)
        A[:m, :k] = _i8(R, m * k).reshape(m, k)
        B[:n, :k] = _i8(R, n * k).reshape(n, k)
        yield f"gemm_int8_{m}_{n}_{k}", "launch_gemm_int8", [In(A), In(B), Out((m, n), np.int32, -3), m, n, k]
    for (m, n, k) in [(33, 17, 5), (70, 4, 2)]:
        yield f"gemm_fp32_{m}_{n}_{k}", "launch_gemm_fp32", [
            In(_f32(R, m * k)), In(_f32(R, k * n)), Out((m, n), np.float32, 9.0, "rel1e-5"), m, n, k]
    # ---- conv helpers
    for gi, g in enumerate(conv_geoms()):
        b, cin, h, w, cout, kh, kw, sh, sw, ph, pw = g
        ho, wo = out_hw(g)
        rows, cols = b * ho * wo, cin * kh * kw
        x8 = _i8(R, b * cin * h * w)
        yield f"im2col_pad_{gi}", "launch_im2col_pad", [
            In(x8), Out((a16(rows), a16(cols)), np.int8, 0x55), b, cin, h, w, kh, kw, sh, sw, ph, pw, ho, wo,
            a16(cols)]
        yield f"im2col_gpu_{gi}", "launch_im2col_gpu", [
            In(x8), Out((rows, cols), np.float32, 7.0), b, cin, h, w, kh, kw, sh, sw, ph, pw, ho, wo]
        go = _f32(R, b * cout * ho * wo)
        yield f"grad_weight_{gi}", "launch_conv_backward_grad_weight", [
            In(x8), In(go), Out((cout * cols,), np.float32, 7.0, "rel1e-5"), b, cin, h, w, cout, kh, kw, sh, sw,
            ph, pw, ho, wo]
        yield f"grad_bias_{gi}", "launch_conv_backward_grad_bias", [
            In(go), Out((cout,), np.float32, 7.0, "rel1e-5"), b, cout, ho, wo]
        wf = _f32(R, cout * cols, 0.1)
        yield f"grad_input_{gi}", "launch_conv_backward_grad_input", [
            In(go), In(wf), Out((b * cin * h * w,), np.float32, 7.0), b, cin, h, w, cout, kh, kw, sh, sw, ph, pw,
            ho, wo]
        wq = np.zeros((a16(cout), a16(cols)), np.int8)
        wq[:cout, :cols] = _i8(R, cout * cols).reshape(cout, cols)
        yield f"grad_input_i8_{gi}", "launch_conv_backward_grad_input_i8", [
            In(go), In(wq), a16(cols), 0.0123, Out((b * cin * h * w,), np.float32, 7.0), b, cin, h, w, cout, kh,
            kw, sh, sw, ph, pw, ho, wo]
        acc = R.integers(-40000, 40000, size=rows * (cout + 3), dtype=np.int64).astype(np.int32)
        bias = _f32(R, cout)
        yield f"conv_epilogue_{gi}", "launch_conv_epilogue", [
            In(acc), In(bias), Out((b * cout * ho * wo,), np.int8, 0x55), cout + 3, 127.0, 50.0, b, cout, ho, wo]
        yield f"epilogue_f32_{gi}", "launch_epilogue_f32", [
            In(acc), cout + 3, 0.000731, Out((b * cout * ho * wo,), np.float32, 7.0), cout, ho, wo,
            b * cout * ho * wo]
    # ---- maxpool
    for (b, c, h, w) in [(2, 3, 6, 8), (1, 5, 2, 30), (3, 2, 16, 80)]:
        x = _i8(R, b * c * h * w, -4, 4)  # many ties
        ny = b * c * (h // 2) * (w // 2)
        yield f"maxpool_fwd_{b}_{c}_{h}_{w}", "launch_maxpool2x2_forward_i8", [
            In(x), Out((ny,), np.int8, 0x55), b, c, h, w]
        yield f"maxpool_bwd_{b}_{c}_{h}_{w}", "launch_maxpool2x2_backward_i8", [
            In(x), In(_f32(R, ny)), Out((x.size,), np.float32, 7.0), b, c, h, w]
    idx = np.array([3, 0, 7, 7, 2], dtype=np.int64)
    yield "maxpool_bwd_idx", "launch_maxpool2x2_backward", [
        In(_f32(R, 5)), In(idx), Out((9,), np.float32, 7.0), 5, 9]
    # ---- BN / quantisation / SE (NCHW with C channels over HW)
    for (b, c, hw) in [(2, 5, 37), (4, 16, 320), (3, 64, 80)]:
        n = b * c * hw
        x = _f32(R, n, 2.0) + np.float32(0.3)
        mean = _f32(R, c, 0.2)
        var = np.abs(_f32(R, c)) + np.float32(0.05)
        gamma, beta = _f32(R, c) + np.float32(1.0), _f32(R, c, 0.1)
        dy = _f32(R, n)
        tag = f"{b}_{c}_{hw}"
        yield f"bn_stats_{tag}", "launch_bn_stats", [
            In(x), b, c, hw, Out((c,), np.float32, 7.0, "rel1e-6"), Out((c,), np.float32, 7.0, "rel1e-5")]
        yield f"bn_apply_{tag}", "launch_bn_apply", [
            In(x), In(mean), In(var), In(gamma), In(beta), 1e-5, Out((n,), np.float32, 7.0), c, hw, n]
        yield f"bn_bwd_sums_{tag}", "launch_bn_bwd_sums", [
            In(dy), In(x), In(mean), In(var), 1e-5, c, hw, n, Out((c,), np.float32, 7.0, "rel1e-5"),
            Out((c,), np.float32, 7.0, "rel1e-5")]
        sdy, sdx = _f32(R, c, 3.0), _f32(R, c, 3.0)
        yield f"bn_bwd_dx_{tag}", "launch_bn_bwd_dx", [
            In(dy), In(x), In(mean), In(var), In(gamma), In(sdy), In(sdx), 1e-5, c, hw, n, b * hw,
            Out((n,), np.float32, 7.0)]
        yield f"reduce_max_abs_{tag}", "launch_reduce_max_abs", [In(x), n, Out((1,), np.float32, 7.0)]
        yield f"max_abs_f32_{tag}", "launch_max_abs_f32", [In(dy), Out((1,), np.float32, 7.0), n]
        s = float(np.abs(x).max() / 127.0)
        yield f"quant_{tag}", "launch_quant_f32_i8", [In(x), n, s, Out((n,), np.int8, 0x55)]
        yield f"relu_quant_{tag}", "launch_relu_quant", [In(x), n, s * 0.7, Out((n,), np.int8, 0x55)]
        q = _i8(R, n)
        q2 = _i8(R, n)
        yield f"dequant_{tag}", "launch_dequant_i8_f32", [In(q), n, 0.0371, Out((n,), np.float32, 7.0)]
        yield f"add_scaled_{tag}", "launch_add_scaled_i8", [In(q), 0.013, In(q2), 0.0071, n,
                                                           Out((n,), np.float32, 7.0)]
        yield f"avgpool_{tag}", "launch_avgpool_hw", [In(x), c, hw, b, Out((b * c,), np.float32, 7.0)]
        yield f"avgpool_bwd_{tag}", "launch_avgpool_hw_backward", [In(_f32(R, b * c)), c, hw, b,
                                                                  Out((n,), np.float32, 7.0)]
        gate = (1.0 / (1.0 + np.exp(-_f32(R, b * c)))).astype(np.float32)
        yield f"mul_gate_{tag}", "launch_mul_gate", [In(x), In(gate), c, hw, n, Out((n,), np.float32, 7.0)]
        yield f"mask_relu_{tag}", "launch_mask_relu_bwd", [In(x), In(dy), n, Out((n,), np.float32, 7.0)]
        yield f"add_{tag}", "launch_add_f32", [In(x), In(dy), n, Out((n,), np.float32, 7.0)]
        yield f"mul_{tag}", "launch_mul_f32", [In(x), In(dy), n, Out((n,), np.float32, 7.0)]
        yield f"zero_{tag}", "launch_zero_f32", [Out((n,), np.float32, 7.0), n]
        yield f"transpose_i8_{tag}", "launch_transpose_i8", [In(q), b * hw, c, Out((n,), np.int8, 0x55)]
        yield f"transpose_f32_{tag}", "cuda_transpose_f32", [In(x), Out((n,), np.float32, 7.0), b * hw, c]
        yield f"f2h_{tag}", "cuda_float_to_half", [In(x), Out((n,), np.uint16, 0x5555), n]
        acc32 = R.integers(-9000, 9000, size=n, dtype=np.int64).astype(np.int32)
        yield f"grad_accum_{tag}", "launch_grad_accum_i32", [
            In(acc32), Out((n,), np.float32, _f32(R, n), "inout"), 0.0173, n]
        yield f"sum_sq_add_{tag}", "launch_sum_sq_add_f32", [In(x), Out((1,), np.float64, 0.5, "rel1e-12"), n]
    for (b, c, h, w) in [(2, 16, 2, 21), (3, 8, 1, 20), (2, 4, 3, 7)]:
        n = b * c * h * w
        x = _f32(R, n)
        yield f"meanpool_h_{b}_{c}_{h}_{w}", "launch_meanpool_h", [In(x), c, h, w, b,
                                                                   Out((b * w * c,), np.float32, 7.0)]
        yield f"meanpool_h_bwd_{b}_{c}_{h}_{w}", "launch_meanpool_h_backward", [
            In(_f32(R, b * w * c)), c, h, w, b, Out((n,), np.float32, 7.0)]
    # ---- optimiser state
    for (rows, col) in [(5, 27), (64, 576), (1, 1)]:
        n = rows * col
        wv = _f32(R, n, 0.05)
        yield f"quantize_pad_{rows}_{col}", "launch_quantize_pad_i8", [
            In(wv), In(np.array([np.abs(wv).max()], np.float32)), Out((1,), np.float32, 7.0),
            Out((a16(rows), a16(col)), np.int8, 0x55), rows, col, a16(col)]
        g = _f32(R, n, 0.01)
        yield f"muon_{rows}_{col}", "launch_muon_step_f32", [
            Out((n,), np.float32, wv, "inout"), In(g), In(np.array([float((g.astype(np.float64) ** 2).sum())])), n,
            5.107e-4, 1.9548e-5, 0.9, float(min(rows, col)), float(max(rows, col)), 10.0, 1]
        yield f"adam_{rows}_{col}", "launch_adam_f32", [
            Out((n,), np.float32, wv, "inout"), In(g), Out((n,), np.float32, _f32(R, n, 1e-3), "inout"),
            Out((n,), np.float32, np.abs(_f32(R, n, 1e-4)), "inout"), n, 5.107e-4, 1.9548e-5, 0.83, 0.9,
            0.999, 1e-8, 1.0 - 0.9 ** 3, 1.0 - 0.999 ** 3]
    yield "scale_vector", "cuda_scale_vector", [Out((1001,), np.float32, _f32(R, 1001), "inout"), 0.37, 1001]
    # ---- fp32 BiLSTM slot kernels
    B, T, D, H = 3, 5, 24, 16
    x = _f32(R, B * T * D)
    wih, whh = _f32(R, 4 * H * D, 0.2), _f32(R, 4 * H * H, 0.2)
    bih, bhh = _f32(R, 4 * H, 0.1), _f32(R, 4 * H, 0.1)
    gates = _f32(R, T * B * 4 * H)
    c_tr, h_tr = _f32(R, T * B * H), _f32(R, T * B * H)
    for slot, rev in [(0, 0), (2, 0), (3, 1)]:
        yield f"lstm_fwd_{slot}_{rev}", "launch_lstm_fwd_step", [
            In(x), In(wih), In(bih), In(whh), In(bhh), Out((T * B * 4 * H,), np.float32, gates, "inout_rel1e-5"),
            Out((T * B * H,), np.float32, c_tr, "inout_rel1e-5"), Out((T * B * H,), np.float32, h_tr, "inout_rel1e-5"),
            B, T, D, H, slot, rev]
    sig = (1.0 / (1.0 + np.exp(-gates))).astype(np.float32)
    for slot in (0, 3):
        yield f"lstm_bwd_cell_{slot}", "launch_lstm_bwd_cell", [
            In(_f32(R, T * B * H)), In(sig), In(c_tr), In(_f32(R, B * H)), In(_f32(R, B * H)),
            Out((T * B * 4 * H,), np.float32, 7.0, "rel1e-5"), Out((B * H,), np.float32, 7.0, "rel1e-5"), B, H, slot]
    dg = _f32(R, T * B * 4 * H)
    for slot, rev in [(0, 0), (4, 1)]:
        yield f"lstm_bwd_rec_{slot}_{rev}", "launch_lstm_bwd_rec", [
            In(dg), In(wih), In(whh), Out((B * T * D,), np.float32, 0.0, "rel1e-5"),
            Out((B * H,), np.float32, 7.0, "rel1e-5"), B, T, D, H, slot, rev]
    for rev, accum in [(0, 0), (1, 1)]:
        yield f"lstm_wgrad_ih_{rev}_{accum}", "launch_lstm_wgrad_ih", [
            In(dg), In(x), Out((4 * H * D,), np.float32, 0.25, "rel1e-5"), B, T, D, H, rev, accum]
    yield "lstm_wgrad_hh", "launch_lstm_wgrad_hh", [
        In(dg), In(h_tr), Out((4 * H * H,), np.float32, 0.25, "rel1e-5"), B, T, H, 1]
    yield "lstm_bgrad", "launch_lstm_bgrad", [
        In(dg), Out((4 * H,), np.float32, 0.5, "rel1e-5"), Out((4 * H,), np.float32, 0.25, "rel1e-5"), B, T, H, 0]


def run_case(be, fn, args):
    """Calls `fn` through backend adapter `be`; returns the list of outputs."""
    import ctypes as C
    call_args, outs, keep = [], [], []
    for a in args:
        if isinstance(a, In):
            h = be.buf(a.a)
            keep.append(h)  # the buffer must outlive the call
            call_args.append(be.ptr(h))
        elif isinstance(a, Out):
            if isinstance(a.fill, np.ndarray):
                init = np.ascontiguousarray(a.fill.astype(a.dtype).reshape(a.shape))
            else:
                init = np.full(a.shape, a.fill, dtype=a.dtype)
            h = be.buf(init)
            call_args.append(be.ptr(h))
            outs.append((h, a))
        else:
            call_args.append(a)
    f = getattr(be.L, fn)
    f(*call_args, be.stream) if fn not in ("maxpool2x2_backward_host",) else f(*call_args)
    be.sync()
    return [(be.get(h), spec) for h, spec in outs]


def compare_outputs(got, want) -> list[str]:
    msgs = []
    for i, ((g, spec), (w, _)) in enumerate(zip(got, want)):
        tol = spec.tol.replace("inout_", "").replace("inout", "exact")
        if tol == "exact":
            if not np.array_equal(g, w, equal_nan=True):
                nd = int((g != w).sum())
                msgs.append(f"out{i}: {nd}/{g.size} elements differ")
        else:
            r = float(tol.replace("rel", ""))
            gd, wd = g.astype(np.float64), w.astype(np.float64)
            d = float(np.abs(gd - wd).max()) if g.size else 0.0
            lim = r * max(1.0, float(np.abs(wd).max()))
            if not d <= lim:
                msgs.append(f"out{i}: max diff {d:.3g} > {lim:.3g}")
    return msgs
