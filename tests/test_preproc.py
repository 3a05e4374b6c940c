"""Line-image preprocessing (load_image_q, src/main.rs:218-239): the device
kernel (include/trba_preproc.h, trba_b200.preproc) against the CPU
restatement (oracle/preproc_oracle.py), bit for bit, and the restatement
against the reference's own arithmetic on cases it decides by itself (exact
sizes, white canvas, target sizes).  The resize is the `image` crate's
(0.24.9), which is not vendored: no golden vectors pin it."""
import ctypes as C
import sys

import numpy as np
import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))
import preproc_oracle as po  # noqa: E402

F32 = np.float32

SHAPES = [(1, 1), (32, 160), (16, 80), (100, 1500), (200, 100), (47, 333), (64, 2000), (5, 700), (31, 159),
          (33, 161), (3, 7), (128, 640), (40, 5000)]


def rgb(rng, h, w):
    return rng.integers(0, 256, (h, w, 3), dtype=np.uint8)


# ------------------------------------------------------------- oracle (CPU) --
def test_round_half_away_is_exact():
    x = np.array([0.5, -0.5, 1.5, 2.5, -2.5, 0.49999997, -0.49999997, 8388607.5, 0.0, -0.0], F32)
    want = np.array([1, -1, 2, 3, -3, 0, 0, 8388608, 0, 0], F32)
    assert np.array_equal(po.round_half_away(x), want)


@pytest.mark.parametrize("h0,w0,want", [((100), (1500), (160, 11)), (200, 100, (16, 32)), (1, 1, (32, 32)),
                                        (32, 160, (160, 32)), (64, 320, (160, 32)), (10, 5000, (160, 1))])
def test_target_size(h0, w0, want):
    """scale = min(img_h / h0, img_w / w0) in f32, nw / nh rounded half away, >= 1."""
    assert po.target_size(h0, w0, 32, 160) == want


def test_exact_size_is_a_copy_then_quantised():
    img = rgb(np.random.default_rng(1), 32, 160)
    q = po.load_image_q(img, 32, 160)
    assert np.array_equal(q, po.quantize_pixels(img).reshape(-1))


def test_quantisation_endpoints():
    """((p / 255) * 2 - 1) * 127: 0 -> -127, 255 -> 127, 128 and 127 -> 0
    (+-0.498), 129 -> 1 (1.49 rounds down), 191 -> 63 (63.25)."""
    q = po.quantize_pixels(np.array([0, 255, 128, 127, 129, 191], np.uint8))
    assert q.tolist() == [-127, 127, 0, 0, 1, 63]


def test_white_canvas_outside_the_resized_image():
    img = rgb(np.random.default_rng(2), 100, 1500)  # -> 160 x 11, centred: rows 10..20
    q = po.load_image_q(img, 32, 160).reshape(32, 160, 3)
    nw, nh = po.target_size(100, 1500, 32, 160)
    y0 = (32 - nh) // 2
    assert (q[:y0] == 127).all() and (q[y0 + nh:] == 127).all()
    tall = po.load_image_q(rgb(np.random.default_rng(3), 200, 100), 32, 160).reshape(32, 160, 3)
    assert (tall[:, 16:] == 127).all()


def test_constant_image_stays_constant():
    for shape in [(100, 1500), (7, 3), (300, 20)]:
        img = np.full(shape + (3,), 200, np.uint8)
        nw, nh = po.target_size(shape[0], shape[1], 32, 160)
        out = po.resize_triangle(img, nw, nh)
        assert (out == 200).all()


def test_library_exports_the_entry_point(lib):
    assert hasattr(lib, "trba_preprocess_lines")


# --------------------------------------------------------------- device --
@pytest.mark.gpu
@pytest.mark.parametrize("img_h,img_w", [(32, 160), (32, 64), (32, 256)])
def test_device_matches_oracle(img_h, img_w, lib, cuda):
    import trba_b200.preproc as pp
    rng = np.random.default_rng(img_w)
    imgs = [rgb(rng, h, w) for h, w in SHAPES]
    got = pp.preprocess_lines(imgs, img_h, img_w).cpu().numpy()
    for i, im in enumerate(imgs):
        want = po.load_image_q(im, img_h, img_w)
        assert np.array_equal(got[i], want), f"image {i} {im.shape}"


@pytest.mark.gpu
def test_device_line_images(lib, cuda):
    """A batch shaped like handwriting lines: height 40..160, width 4..16x height,
    dark strokes on light paper."""
    import trba_b200.preproc as pp
    rng = np.random.default_rng(7)
    imgs = []
    for _ in range(24):
        h = int(rng.integers(40, 160))
        w = int(h * rng.uniform(4, 16))
        im = np.full((h, w, 3), 235, np.uint8)
        strokes = rng.random((h, w)) < 0.08
        im[strokes] = rng.integers(0, 80, (int(strokes.sum()), 1), dtype=np.uint8)
        imgs.append(im)
    got = pp.preprocess_lines(imgs, 32, 160).cpu().numpy()
    for i, im in enumerate(imgs):
        assert np.array_equal(got[i], po.load_image_q(im, 32, 160)), f"image {i} {im.shape}"


@pytest.mark.gpu
def test_device_arguments(lib, cuda):
    import torch
    out = torch.empty(16, dtype=torch.int8, device=cuda)
    assert lib.trba_preprocess_lines(None, None, None, None, 0, 32, 160, None, None) == 0  # empty batch
    assert lib.trba_preprocess_lines(None, None, None, None, 1, 32, 160, C.c_void_p(out.data_ptr()), None) == -1
