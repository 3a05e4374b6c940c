"""The conv forward as an implicit GEMM (trba_conv_gemm_int8_implicit) against
the reference's im2col + GEMM pair (launch_im2col_pad, launch_gemm_int8 of the
oracle, itself pinned to the reference's CPU backend).

The GEMM gathers each output pixel's receptive field from the activations
into its shared-memory stages in (ky, kx, ci) order; integer accumulation does
not depend on the order of the K terms, so the s32 accumulators must equal the
reference's bit for bit on every conv shape of the model and on ragged ones
(a partial last row tile, N not a multiple of the tile width, two N tiles,
Cin up to 512, asymmetric kernels, strides and padding)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

A16 = lambda x: (x + 15) & ~15  # noqa: E731

# (B, Cin, H, W, Cout, kh, kw, sh, sw, ph, pw)
SHAPES = [
    (2, 16, 32, 160, 32, 3, 3, 1, 1, 1, 1),    # stem.3
    (3, 32, 16, 80, 64, 3, 3, 2, 2, 1, 1),     # layer1.0.conv1 (stride 2)
    (3, 32, 16, 80, 64, 1, 1, 2, 2, 0, 0),     # layer1.0.downsample (1x1 stride 2)
    (4, 64, 8, 40, 64, 3, 3, 1, 1, 1, 1),      # layer2.x
    (4, 64, 8, 40, 128, 3, 3, 2, 2, 1, 1),     # layer3.0.conv1
    (4, 64, 8, 40, 128, 1, 1, 2, 2, 0, 0),     # layer3.0.downsample
    (5, 128, 4, 20, 128, 3, 3, 1, 1, 1, 1),    # layer3/4
    (5, 128, 4, 20, 128, 2, 2, 2, 1, 0, 1),    # conv_out.0 (2x2, stride (2, 1), pad (0, 1))
    (5, 128, 2, 21, 128, 2, 2, 1, 1, 0, 0),    # conv_out.3
    (3, 16, 7, 9, 48, 3, 3, 1, 1, 1, 1),       # Cout 48 (partial 64-wide tile), 7x9 planes
    (2, 32, 5, 6, 200, 3, 3, 2, 2, 1, 1),      # Cout 200: a 256-wide tile, odd planes
    (1, 256, 6, 10, 64, 3, 3, 1, 1, 1, 1),     # K = 2304
    (1, 512, 3, 5, 32, 3, 3, 1, 1, 1, 1),      # K = 4608
    (2, 16, 6, 5, 16, 3, 2, 1, 1, 1, 0),       # asymmetric kernel and padding
    (2, 32, 6, 9, 32, 3, 3, 1, 1, 0, 2),       # padding 0 on one axis, 2 on the other
    (2, 64, 9, 6, 32, 3, 3, 2, 1, 1, 1),       # stride (2, 1)
    (1, 16, 1, 1, 16, 3, 3, 1, 1, 1, 1),       # a single pixel: eight of nine taps in the padding
]


def _out_hw(h, w, kh, kw, sh, sw, ph, pw):
    return (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1


def _reference(oracle, x, wq, wld, B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo):
    rows = B * ho * wo
    k = cin * kh * kw
    col = np.zeros((A16(rows), A16(k)), np.int8)
    oracle.launch_im2col_pad(x.ctypes.data, col.ctypes.data, B, cin, h, w, kh, kw, sh, sw, ph, pw, ho, wo, A16(k),
                             None)
    acc = np.zeros((rows, cout), np.int32)
    oracle.launch_gemm_int8(col.ctypes.data, wq.ctypes.data, acc.ctypes.data, rows, cout, k, None)
    return acc


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "b{}_c{}_{}x{}_o{}_k{}x{}_s{}{}_p{}{}".format(*s))
def test_implicit_conv_gemm_matches_im2col_gemm(shape, lib, cuda, oracle):
    import torch
    B, cin, h, w, cout, kh, kw, sh, sw, ph, pw = shape
    ho, wo = _out_hw(h, w, kh, kw, sh, sw, ph, pw)
    rng = np.random.default_rng(sum(shape) + 7)
    x = rng.integers(-127, 128, (B, cin, h, w)).astype(np.int8)
    k = cin * kh * kw
    wld = A16(k)
    wq = np.zeros((A16(cout), wld), np.int8)
    wq[:cout, :k] = rng.integers(-127, 128, (cout, k))
    want = _reference(oracle, x, wq, wld, B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo)
    d_x = torch.from_numpy(x).cuda()
    d_w = torch.from_numpy(wq).cuda()
    d_acc = torch.full((B * ho * wo, cout), -(2 ** 31), dtype=torch.int32, device="cuda")
    for _ in range(2):  # a second call reuses the per-device buffer
        rc = lib.trba_conv_gemm_int8_implicit(C.c_void_p(d_x.data_ptr()), C.c_void_p(d_w.data_ptr()), wld,
                                              C.c_void_p(d_acc.data_ptr()), B, cin, h, w, cout, kh, kw, sh, sw, ph,
                                              pw, ho, wo, None)
        assert rc == 0, lib.trba_last_error_string()
        got = d_acc.cpu().numpy()
        assert np.array_equal(got, want), f"{int((got != want).sum())} of {want.size} accumulators differ"
    assert lib.trba_tc_error_poll(1) == 0
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


def test_implicit_conv_gemm_refuses_unsupported_convs(lib, cuda):
    """Cin must be a power of two >= 16 (whole 16-byte channel runs per tap);
    the call reports the refusal instead of computing."""
    import torch
    x = torch.zeros(2 * 24 * 8 * 8, dtype=torch.int8, device="cuda")
    wq = torch.zeros(16 * A16(24 * 9), dtype=torch.int8, device="cuda")
    acc = torch.zeros(2 * 8 * 8 * 16, dtype=torch.int32, device="cuda")
    rc = lib.trba_conv_gemm_int8_implicit(C.c_void_p(x.data_ptr()), C.c_void_p(wq.data_ptr()), A16(24 * 9),
                                          C.c_void_p(acc.data_ptr()), 2, 24, 8, 8, 16, 3, 3, 1, 1, 1, 1, 8, 8, None)
    assert rc == -1
    assert "unsupported conv" in lib.trba_last_error_string().decode()
    lib.trba_clear_error()
