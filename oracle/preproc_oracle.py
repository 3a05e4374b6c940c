"""CPU restatement of the reference's line-image preprocessing (test
infrastructure: the checker of the device kernel, never the product path).

Reference: `load_image_q` (src/main.rs:218-239): RGB8 -> aspect-preserving
resize with `image::imageops::resize(.., FilterType::Triangle)` -> white
canvas (aligned left, centred vertically) -> ((p / 255) * 2 - 1) * 127,
rounded, clamped to +-127, int8, in the reference's interleaved [y][x][rgb]
byte order (which the model then reads as its [3, H, W] input).

The resize lives in the third-party crate `image` 0.24.9 (Cargo.lock), which
is not vendored with the reference; this file restates its published
separable-resampling algorithm: a vertical pass into an f32 image, then a
horizontal pass rounded to u8.  For output coordinate o over an input of
length n resized to m: ratio = n / m, sratio = max(ratio, 1), support =
sratio (triangle filter support 1), centre = (o + 0.5) * ratio, taps
i in [clamp(floor(centre - support), 0, n - 1), clamp(ceil(centre +
support), left + 1, n)), weight = tri((i - (centre - 0.5)) / sratio) with
tri(x) = max(1 - |x|, 0), normalised by their f32 sum; each output is the
sequential f32 sum of pixel * weight (a rounded multiply, then a rounded
add); the horizontal pass clamps to [0, 255] and rounds half away from
zero.  Equal source and target sizes copy the image.  Every operation is
single precision, as in the crate.  No golden vectors exist for this step
(the reference has no test of it), so parity with the crate itself is
unpinned; the device kernel is pinned to this restatement bit for bit.
"""
from __future__ import annotations

import numpy as np

F = np.float32


def round_half_away(x: np.ndarray) -> np.ndarray:
    """Round half away from zero, exactly, for |x| < 2**23 (f32)."""
    x = np.asarray(x, dtype=F)
    a = np.abs(x)
    fl = np.floor(a)
    r = fl + (a - fl >= F(0.5)).astype(F)
    return np.copysign(r, x).astype(F)


def _weights(o: int, n: int, m: int):
    ratio = F(n) / F(m)
    sratio = ratio if ratio >= F(1.0) else F(1.0)
    support = F(1.0) * sratio
    centre = (F(o) + F(0.5)) * ratio
    left = int(np.floor(centre - support))
    left = min(max(left, 0), n - 1)
    right = int(np.ceil(centre + support))
    right = min(max(right, left + 1), n)
    c = centre - F(0.5)
    ws = []
    s = F(0.0)
    for i in range(left, right):
        x = (F(i) - c) / sratio
        ax = abs(x)
        w = F(1.0) - ax if ax < F(1.0) else F(0.0)
        ws.append(F(w))
        s = F(s + F(w))
    return left, [F(w / s) for w in ws]


def resize_triangle(img: np.ndarray, nw: int, nh: int) -> np.ndarray:
    """image 0.24.9 `resize` with FilterType::Triangle on an [h, w, 3] u8 image."""
    h0, w0, _ = img.shape
    if (nw, nh) == (w0, h0):
        return img.copy()
    src = img.astype(F)
    tmp = np.empty((nh, w0, 3), F)
    for y in range(nh):
        left, ws = _weights(y, h0, nh)
        t = np.zeros((w0, 3), F)
        for k, w in enumerate(ws):
            t = (t + src[left + k] * w).astype(F)
        tmp[y] = t
    out = np.empty((nh, nw, 3), np.uint8)
    for x in range(nw):
        left, ws = _weights(x, w0, nw)
        t = np.zeros((nh, 3), F)
        for k, w in enumerate(ws):
            t = (t + tmp[:, left + k] * w).astype(F)
        out[:, x] = round_half_away(np.clip(t, F(0.0), F(255.0))).astype(np.uint8)
    return out


def target_size(h0: int, w0: int, img_h: int, img_w: int):
    """(nw, nh) of the reference: f32 scale = min(img_h / h0, img_w / w0)."""
    scale = min(F(img_h) / F(max(h0, 1)), F(img_w) / F(max(w0, 1)))
    nw = max(round_half_away(F(w0) * scale), F(1.0))
    nh = max(round_half_away(F(h0) * scale), F(1.0))
    return int(nw), int(nh)


def quantize_pixels(buf: np.ndarray) -> np.ndarray:
    """((p / 255) * 2 - 1) * 127, rounded half away from zero, clamped to +-127."""
    v = (((buf.astype(F) / F(255.0)) * F(2.0) - F(1.0)) * F(127.0)).astype(F)
    return np.clip(round_half_away(v), -127, 127).astype(np.int8)


def load_image_q(img: np.ndarray, img_h: int, img_w: int) -> np.ndarray:
    """The reference's preprocessing of one decoded RGB8 image [h0, w0, 3]:
    int8 [img_h * img_w * 3] in [y][x][rgb] order."""
    h0, w0, _ = img.shape
    nw, nh = target_size(h0, w0, img_h, img_w)
    resized = resize_triangle(img, nw, nh)
    buf = np.full((img_h, img_w, 3), 255, np.uint8)
    y0 = max(img_h - nh, 0) // 2
    buf[y0:y0 + nh, :nw] = resized
    return quantize_pixels(buf).reshape(-1)
