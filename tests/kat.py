"""Known-answer cases of the reference's own unit tests, restated in numpy.

Inputs come from the reference's deterministic generator det(i, seed)
(src/tests.rs:39-43); shapes, seeds and scale factors are those of the
reference tests cited on each case.  The expected outputs are the
reference tests' own naive formulas, restated here; tests/golden/make_golden.py
also runs the reference's CPU backend (oracle/_ref) on the same inputs and
stores its outputs in tests/golden/ref_kat.npz.
"""
from __future__ import annotations

import numpy as np

U64 = np.uint64


def det(n: int, seed: int) -> np.ndarray:
    """src/tests.rs:39-43, vectorised: float32 in [-1, 1]."""
    i = np.arange(n, dtype=U64)
    with np.errstate(over="ignore"):
        x = (i * U64(2654435761)) ^ U64(seed)
        x = x * U64(6364136223846793005) + U64(1442695040888963407)
    hi = (x >> U64(33)).astype(np.float64).astype(np.float32)
    return (hi / np.float32(2147483648.0)) * np.float32(2.0) - np.float32(1.0)


def det_i8(n: int, seed: int, mul: float = 100.0) -> np.ndarray:
    """Rust `(det(i, seed) * mul) as i8` (truncate toward zero, saturate)."""
    v = det(n, seed) * np.float32(mul)
    return np.clip(np.trunc(v), -128, 127).astype(np.int8)


def det_i32(n: int, seed: int, mul: float) -> np.ndarray:
    v = det(n, seed) * np.float32(mul)
    return np.trunc(v).astype(np.int32)


def a16(x: int) -> int:
    return (x + 15) & ~15


def pad2(x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """pad_to_multiple_i8 (src/backend.rs:287-296): zero-pad to multiples of 16."""
    out = np.zeros((a16(rows), a16(cols)), dtype=x.dtype)
    out[:rows, :cols] = x.reshape(rows, cols)
    return out


# ---------------------------------------------------------------- cases --
# src/tests.rs:72-103 (int8_gemm_matches_naive_including_unpadded_shapes)
GEMM_SHAPES = [(16, 16, 16), (17, 5, 3), (100, 33, 27), (256, 192, 512)]


def gemm_case(m, n, k):
    a = det_i8(m * k, 1).reshape(m, k)
    b = det_i8(n * k, 2).reshape(n, k)
    want = a.astype(np.int64) @ b.astype(np.int64).T
    return a, b, want.astype(np.int32)


def ref_im2col(inp, b, c, h, w, kh, kw, sh, sw, ph, pw):
    """src/tests.rs:159-190, compact [rows, c*kh*kw]."""
    ho = (h + 2 * ph - kh) // sh + 1
    wo = (w + 2 * pw - kw) // sw + 1
    x = np.zeros((b, c, h + 2 * ph, w + 2 * pw), dtype=inp.dtype)
    x[:, :, ph:ph + h, pw:pw + w] = inp.reshape(b, c, h, w)
    cols = np.empty((b, ho, wo, c, kh, kw), dtype=inp.dtype)
    for i in range(kh):
        for j in range(kw):
            cols[:, :, :, :, i, j] = x[:, :, i:i + sh * ho:sh, j:j + sw * wo:sw].transpose(0, 2, 3, 1)
    return cols.reshape(b * ho * wo, c * kh * kw), ho, wo


# src/tests.rs:192-228
IM2COL_CASE = (3, 5, 9, 11, 3, 2, 1)  # b, c, h, w, k, s, p (seed 7)

# src/tests.rs:233-264 (conv2d.rs:24-25: ACC_DIVISOR 127, OUT_MULTIPLIER 50)
EPILOGUE_CASE = (2, 5, 3, 4)
ACC_DIVISOR, OUT_MULTIPLIER = np.float32(127.0), np.float32(50.0)


def conv_epilogue_ref(acc, bias, ld, b, c, ho, wo):
    hw = ho * wo
    out = np.empty(b * c * hw, dtype=np.int8)
    i = np.arange(b * c * hw)
    bi, oc, p = i // (c * hw), (i // hw) % c, i % hw
    v = acc[(bi * hw + p) * ld + oc].astype(np.float32) / ACC_DIVISOR + bias[oc]
    v = np.clip(np.maximum(v, np.float32(0)) * OUT_MULTIPLIER, -127, 127).astype(np.float32)
    out[:] = np.rint(v).astype(np.int8)  # the test uses round(); values .5 do not occur here
    return out


def shape(b, cin, h, w, cout, k, s, p):
    """src/tests.rs:277-285: ConvShape."""
    return dict(b=b, cin=cin, h=h, w=w, cout=cout, kh=k, kw=k, sh=s, sw=s, ph=p, pw=p,
                ho=(h + 2 * p - k) // s + 1, wo=(w + 2 * p - k) // s + 1)


# src/tests.rs:373-400, 434-459, 402-432, 572-636
GRAD_W_SHAPES = [shape(2, 3, 8, 7, 5, 3, 1, 1), shape(1, 4, 6, 6, 8, 3, 2, 1), shape(3, 2, 5, 5, 3, 1, 1, 0)]
GRAD_IN_SHAPES = [shape(2, 3, 7, 6, 4, 3, 1, 1), shape(1, 2, 8, 8, 3, 3, 2, 1), shape(2, 2, 4, 9, 2, 1, 1, 0)]
GRAD_IN_I8_SHAPES = GRAD_IN_SHAPES + [shape(1, 4, 5, 5, 17, 3, 1, 1)]
GRAD_BIAS_SHAPE = shape(4, 3, 6, 5, 7, 3, 1, 1)


def ref_grad_w(s, inp, go):
    """src/tests.rs:287-332: go_mat^T @ col in float64 (the test's float32
    accumulation agrees to its 1e-3 tolerance)."""
    col, ho, wo = ref_im2col(inp, s["b"], s["cin"], s["h"], s["w"], s["kh"], s["kw"], s["sh"], s["sw"],
                             s["ph"], s["pw"])
    gom = go.reshape(s["b"], s["cout"], ho * wo).transpose(0, 2, 1).reshape(-1, s["cout"])
    return (gom.astype(np.float64).T @ col.astype(np.float64)).astype(np.float32).ravel()


def ref_grad_input(s, go, weight):
    """src/tests.rs:334-370, via a transposed convolution in float64."""
    b, cin, h, w, cout = s["b"], s["cin"], s["h"], s["w"], s["cout"]
    kh, kw, sh, sw, ph, pw, ho, wo = s["kh"], s["kw"], s["sh"], s["sw"], s["ph"], s["pw"], s["ho"], s["wo"]
    W = weight.reshape(cout, cin, kh, kw).astype(np.float64)
    g = go.reshape(b, cout, ho, wo).astype(np.float64)
    out = np.zeros((b, cin, h + 2 * ph + sh * kh, w + 2 * pw + sw * kw))
    for i in range(kh):
        for j in range(kw):
            contrib = np.einsum("bohw,oc->bchw", g, W[:, :, i, j])
            out[:, :, i:i + sh * ho:sh, j:j + sw * wo:sw] += contrib
    return out[:, :, ph:ph + h, pw:pw + w].astype(np.float32).ravel()


def host_requantize(w):
    """ConvQat::requantize (src/qnet.rs:316-331): f32 division, round half away."""
    mx = np.float32(np.abs(w).max()) if w.size else np.float32(0)
    ws = np.float32(mx / np.float32(127.0)) if mx > 0 else np.float32(1.0)
    q = np.clip(w / ws, -127, 127).astype(np.float32)
    q = (np.sign(q) * np.floor(np.abs(q) + np.float32(0.5))).astype(np.int8)
    return q, ws


# src/tests.rs:473-532 (maxpool_i8_on_device_matches_host_index_reference)
MAXPOOL_CASES = [(1, 1, 2, 2, False), (2, 3, 6, 8, False), (1, 128, 4, 16, False), (2, 2, 4, 4, True)]


def maxpool_input(b, c, h, w, ties):
    n = b * c * h * w
    if ties:
        return ((np.arange(n) // (h * w)) * 3 + 1).astype(np.int8)
    return det_i8(n, 47)


def maxpool_with_indices(x, b, c, h, w):
    """conv2d::maxpool2x2_with_indices semantics: first strict maximum."""
    x = x.reshape(b * c, h, w)
    ho, wo = h // 2, w // 2
    y = np.empty((b * c, ho, wo), dtype=np.int8)
    idx = np.empty((b * c, ho, wo), dtype=np.int64)
    for bc in range(b * c):
        for oh in range(ho):
            for ow in range(wo):
                best, bi = None, 0
                for di, dj in ((0, 0), (0, 1), (1, 0), (1, 1)):
                    v = x[bc, 2 * oh + di, 2 * ow + dj]
                    if best is None or v > best:
                        best, bi = v, (2 * oh + di) * w + 2 * ow + dj
                y[bc, oh, ow] = best
                idx[bc, oh, ow] = bc * h * w + bi
    return y.ravel(), idx.ravel()


# src/tests.rs:534-568: literal golden vector
MAXPOOL_ZERO_INPUT = np.array([1, 9, 2, 2, -3, -3, -3, -3], dtype=np.int8)
MAXPOOL_ZERO_WANT = np.array([0.0, 1.5, 0.0, 0.0, 1.5, 0.0, 0.0, 0.0], dtype=np.float32)

# src/tests.rs:640-690
REQUANT_SHAPES = [(4, 27), (16, 16), (17, 5), (64, 2048), (1, 1)]

# src/tests.rs:693-741
ADAM_N = 1000
ADAM_HP = dict(lr=5.107e-4, wd=1.9548e-5, clip=0.83, b1=0.9, b2=0.999, eps=1e-8,
               bc1=1.0 - 0.9 ** 7, bc2=1.0 - 0.999 ** 7)


def adam_inputs():
    n = ADAM_N
    return (det(n, 37) * np.float32(0.2), det(n, 41) * np.float32(3.0),
            det(n, 43) * np.float32(0.01), np.abs(det(n, 47)) * np.float32(0.01))


def adam_host(p, g, m, v, lr, wd, clip, b1, b2, eps, bc1, bc2):
    """The test's host replay of src/opt.rs arithmetic (f64 intermediates)."""
    p, m, v = p.copy(), m.copy(), v.copy()
    gi = (g.astype(np.float64) * clip).astype(np.float32).astype(np.float64) + wd * p.astype(np.float64)
    m[:] = (b1 * m.astype(np.float64) + (1.0 - b1) * gi).astype(np.float32)
    v[:] = (b2 * v.astype(np.float64) + (1.0 - b2) * gi * gi).astype(np.float32)
    mh = m.astype(np.float64) / bc1
    vh = v.astype(np.float64) / bc2
    p -= (lr * mh / (np.sqrt(vh) + eps)).astype(np.float32)
    return p, m, v
