"""The INT8 operator API (LinearInt8 of src/linear.rs, LSTMInt8 / BiLSTMInt8
of src/bilstm.rs): libtrba_b200's device-resident operators
(include/trba_ops.h, trba_b200.ops) against the numpy oracle
(oracle/ops_oracle.py), and the oracle against the reference's own tests for
these layers (src/tests.rs:553-615, restated)."""
import ctypes as C
import sys

import numpy as np
import pytest

from conftest import REPO
from kat import det, det_i8

sys.path.insert(0, str(REPO / "oracle"))
import ops_oracle as oo  # noqa: E402

F32 = np.float32


def glorot(rng, fan_in, fan_out, n):
    lim = np.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-lim, lim, n).astype(F32)


# ------------------------------------------------------------- oracle (CPU) --
def test_oracle_linear_forward_is_the_int8_product():
    """src/tests.rs:553-571: forward == sum_i inp[r,i] * weight_int8[o,i]."""
    rng = np.random.default_rng(1)
    lin = oo.LinearInt8(glorot(rng, 20, 7, 140), np.zeros(7, F32), 20, 7)
    inp = det_i8(5 * 20, 59)
    out = lin.forward(inp).reshape(5, 7)
    want = inp.reshape(5, 20).astype(np.int64) @ lin.weight_int8.reshape(7, 20).astype(np.int64).T
    assert np.array_equal(out, want)


def test_oracle_linear_backward_matches_reference_test():
    """src/tests.rs:573-615, restated on the oracle with its tolerance."""
    w = (det(4 * 6, 61) * F32(0.5)).astype(F32)
    lin = oo.LinearInt8(w, np.zeros(4, F32), 6, 4)
    rows = 3
    inp = det(rows * 6, 67)
    out = np.array([sum(inp[r * 6 + k] * w[o * 6 + k] for k in range(6)) for r in range(rows) for o in range(4)],
                   F32)
    go = (F32(2.0) * out / F32(rows)).astype(F32)
    before = lin.weight_f32.copy()
    clip = lin.backward(inp, go, 1.0, 0.0)
    for o in range(4):
        for i in range(6):
            g = F32(0.0)
            for r in range(rows):
                g = F32(g + go[r * 4 + o] * inp[r * 6 + i])
            g = F32(g / rows)
            want = before[o * 6 + i] - 1.0 * clip * g
            tol = 1e-5 * max(abs(want), 1.0) + 1e-4
            assert abs(lin.weight_f32[o * 6 + i] - want) < tol


def test_oracle_quantize_rounds_half_away_and_handles_zero():
    w = np.array([127.0, 63.5, -63.5, 0.5, -0.5, 1.5, -2.5, 0.0], F32)
    assert oo.quantize(w).tolist() == [127, 64, -64, 1, -1, 2, -3, 0]   # scale 1.0
    assert oo.quantize(np.zeros(5, F32)).tolist() == [0] * 5            # scale 1 when max is 0
    assert oo.LSTMInt8.quantize_h(np.array([12.7, -0.05, 0.05, 100.0], F32)).tolist() == [127, -1, 1, 127]


def test_oracle_lstm_step_matches_f64_formula():
    rng = np.random.default_rng(2)
    I, H, B = 24, 8, 5
    l = oo.LSTMInt8(glorot(rng, I, 4 * H, 4 * H * I), glorot(rng, H, 4 * H, 4 * H * H),
                    rng.normal(0, 0.1, 4 * H).astype(F32), I, H)
    x = rng.integers(-127, 128, B * I).astype(np.int8)
    h0 = rng.normal(0, 0.5, B * H).astype(F32)
    c0 = rng.normal(0, 0.5, B * H).astype(F32)
    h, c = l.forward_step(x, h0, c0, B)
    hq = np.clip(np.sign(h0 * 10) * np.floor(np.abs(h0.astype(np.float64) * 10) + 0.5), -127, 127)
    gi = x.reshape(B, I).astype(np.float64) @ l.weight_ih_int8.reshape(4 * H, I).astype(np.float64).T
    gh = hq.reshape(B, H) @ l.weight_hh_int8.reshape(4 * H, H).astype(np.float64).T
    pre = (gi + gh) / 1270.0 + l.bias
    sg = lambda v: 1 / (1 + np.exp(-v))  # noqa: E731
    cc = sg(pre[:, H:2 * H]) * c0.reshape(B, H) + sg(pre[:, :H]) * np.tanh(pre[:, 2 * H:3 * H])
    hh = sg(pre[:, 3 * H:]) * np.tanh(cc)
    assert np.allclose(c.reshape(B, H), cc, atol=1e-5) and np.allclose(h.reshape(B, H), hh, atol=1e-5)


def test_oracle_bilstm_runs_both_directions_forward_in_time():
    """Both directions of BiLSTMInt8::forward step t = 0..T-1 (src/bilstm.rs:
    216-231): with identical weights the two halves of the output agree."""
    rng = np.random.default_rng(3)
    I, H, B, T = 16, 8, 3, 4
    wi, wh = glorot(rng, I, 4 * H, 4 * H * I), glorot(rng, H, 4 * H, 4 * H * H)
    bi = oo.BiLSTMInt8(oo.LSTMInt8(wi, wh, np.zeros(4 * H, F32), I, H), oo.LSTMInt8(wi, wh, np.zeros(4 * H, F32), I, H))
    out = bi.forward(rng.integers(-127, 128, T * B * I).astype(np.int8), B, T).reshape(B, 2 * H)
    assert np.array_equal(out[:, :H], out[:, H:])
    assert np.all(bi.forward(np.zeros(0, np.int8), B, 0) == 0)


# ---------------------------------------------------------- product (GPU) --
def _linear_pair(rng, fi, fo, scale=1.0):
    import trba_b200.ops as ops
    w = (glorot(rng, fi, fo, fi * fo) * F32(scale)).astype(F32)
    b = rng.normal(0, 0.1, fo).astype(F32)
    return ops.LinearInt8(fi, fo, w, b), oo.LinearInt8(w, b, fi, fo)


@pytest.mark.gpu
@pytest.mark.parametrize("fi,fo,rows", [(20, 7, 5), (1, 1, 1), (33, 17, 3), (512, 512, 300), (512, 192, 48)])
def test_linear_forward_and_weights_match_oracle(fi, fo, rows, lib, cuda):
    rng = np.random.default_rng(fi * 1000 + fo)
    dev, orc = _linear_pair(rng, fi, fo)
    assert np.array_equal(dev.weight_int8, orc.weight_int8)
    inp = det_i8(rows * fi, 59)
    assert np.array_equal(dev.forward(inp), orc.forward(inp))
    assert dev.param_count() == fi * fo + fo


@pytest.mark.gpu
@pytest.mark.parametrize("grad_scale", [1e-3, 50.0], ids=["unclipped", "clipped"])
def test_linear_backward_matches_oracle(grad_scale, lib, cuda):
    rng = np.random.default_rng(11)
    fi, fo, rows = 64, 40, 37
    dev, orc = _linear_pair(rng, fi, fo)
    for step in range(3):
        inp = rng.normal(0, 1, rows * fi).astype(F32)
        go = (rng.normal(0, 1, rows * fo) * grad_scale).astype(F32)
        c_dev = dev.backward(inp, go, 0.05, 0.9)
        c_orc = orc.backward(inp, go, 0.05, 0.9)
        assert abs(c_dev - c_orc) <= 1e-6 * abs(c_orc), (step, c_dev, c_orc)
        w, q, b, g = dev._state()
        assert np.array_equal(g, orc.grad_f32), "batch-averaged gradient differs"
        if grad_scale < 1:  # clip == 1 on both sides: bit-identical update
            assert np.array_equal(w, orc.weight_f32) and np.array_equal(b, orc.bias)
            assert np.array_equal(q, orc.weight_int8)
        else:
            assert np.allclose(w, orc.weight_f32, rtol=1e-6, atol=1e-7)
            assert np.allclose(b, orc.bias, rtol=1e-6, atol=1e-7)
            assert np.mean(q != orc.weight_int8) < 1e-3


@pytest.mark.gpu
def test_linear_backward_reference_finite_difference_case(lib, cuda):
    """src/tests.rs:573-615 on the device operator."""
    import trba_b200.ops as ops
    w = (det(24, 61) * F32(0.5)).astype(F32)
    lin = ops.LinearInt8(6, 4, w, np.zeros(4, F32))
    rows = 3
    inp = det(rows * 6, 67)
    out = (inp.reshape(rows, 6) @ w.reshape(4, 6).T).astype(F32).ravel()
    go = (F32(2.0) * out / F32(rows)).astype(F32)
    clip = lin.backward(inp, go, 1.0, 0.0)
    got = lin.weight_f32
    g = (go.reshape(rows, 4).T.astype(np.float64) @ inp.reshape(rows, 6).astype(np.float64)) / rows
    want = w.reshape(4, 6) - clip * g
    tol = 1e-5 * np.maximum(np.abs(want), 1.0) + 1e-4
    assert np.all(np.abs(got.reshape(4, 6) - want) < tol)


@pytest.mark.gpu
def test_linear_edge_cases(lib, cuda):
    rng = np.random.default_rng(5)
    dev, _ = _linear_pair(rng, 8, 3)
    before = dev.weight_f32
    assert dev.backward(np.zeros(0, F32), np.zeros(0, F32), 0.1, 0.0) == 0.0       # rows == 0
    assert dev.backward(np.ones(16, F32), np.ones(5, F32), 0.1, 0.0) == 0.0         # grad too short
    assert np.array_equal(dev.weight_f32, before)
    with pytest.raises(ValueError):
        dev.forward(np.zeros(7, np.int8))
    lib.trba_clear_error()
    buf = np.zeros(7, np.int8)
    out = np.zeros(3, np.int32)
    assert lib.trba_linear_int8_forward_host(dev.h, C.c_void_p(buf.ctypes.data), 7, C.c_void_p(out.ctypes.data)) == -1
    assert b"in_features" in lib.trba_last_error_string()
    lib.trba_clear_error()


def _lstm_pair(rng, I, H):
    import trba_b200.ops as ops
    wi, wh = glorot(rng, I, 4 * H, 4 * H * I), glorot(rng, H, 4 * H, 4 * H * H)
    b = rng.normal(0, 0.1, 4 * H).astype(F32)
    return ops.LSTMInt8(I, H, wi, wh, b), oo.LSTMInt8(wi, wh, b, I, H)


@pytest.mark.gpu
@pytest.mark.parametrize("I,H,B", [(24, 8, 5), (128, 64, 48), (512, 64, 17), (3, 1, 1)])
def test_lstm_step_matches_oracle(I, H, B, lib, cuda):
    rng = np.random.default_rng(I + H + B)
    dev, orc = _lstm_pair(rng, I, H)
    st = dev.state()
    assert np.array_equal(st["weight_ih_int8"], orc.weight_ih_int8)
    assert np.array_equal(st["weight_hh_int8"], orc.weight_hh_int8)
    x = rng.integers(-127, 128, B * I).astype(np.int8)
    h0 = rng.normal(0, 0.5, B * H).astype(F32)
    c0 = rng.normal(0, 0.5, B * H).astype(F32)
    assert np.array_equal(dev.i2h_forward(x, B), orc.i2h_forward(x, B))
    hq = orc.quantize_h(h0)
    assert np.array_equal(dev.h2h_forward(hq, B), orc.h2h_forward(hq, B))
    h, c = dev.forward_step(x, h0, c0, B)
    hw, cw = orc.forward_step(x, h0, c0, B)
    assert np.allclose(h, hw, rtol=1e-6, atol=1e-7) and np.allclose(c, cw, rtol=1e-6, atol=1e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("I,H,B,T", [(16, 8, 3, 4), (128, 64, 48, 20), (64, 32, 5, 1), (16, 8, 2, 0)])
def test_bilstm_forward_matches_oracle(I, H, B, T, lib, cuda):
    import trba_b200.ops as ops
    rng = np.random.default_rng(I * T + B)
    f_dev, f_orc = _lstm_pair(rng, I, H)
    b_dev, b_orc = _lstm_pair(rng, I, H)
    x = rng.integers(-127, 128, max(T * B * I, 1)).astype(np.int8)
    got = ops.BiLSTMInt8(f_dev, b_dev).forward(x, B, T)
    want = oo.BiLSTMInt8(f_orc, b_orc).forward(x, B, T)
    assert np.allclose(got, want, rtol=1e-4, atol=1e-5), np.abs(got - want).max()


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(5, 7, 20), (1, 1, 1), (100, 256, 64), (333, 65, 129)])
def test_compact_gemm_matches_oracle(m, n, k, lib, cuda):
    import trba_b200.ops as ops
    rng = np.random.default_rng(m + n + k)
    a = rng.integers(-127, 128, m * k).astype(np.int8)
    b = rng.integers(-127, 128, n * k).astype(np.int8)
    assert np.array_equal(ops.LSTMInt8.gemm_int8(a, b, m, n, k).reshape(m, n), oo.gemm_int8(a, b, m, n, k))
