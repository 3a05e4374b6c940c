"""Regenerate tests/golden/ref_kat.npz from the reference itself.

Runs the reference's own CPU backend (oracle/_ref/libtrba_ref_omp.so, built by
`make -C oracle ref` from the reference's cuda/cpu_backend.cpp) on the
known-answer inputs of the reference's unit tests (tests/kat.py), checks each
output against the test's own expected formula, and stores inputs that are
not det()-derived plus every output.  Needs the reference sources mounted
(this container); the GPU box only reads the committed .npz.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "tests"))
sys.path.insert(0, str(REPO))

import kat  # noqa: E402
from conftest import _typed_cpu_backend  # noqa: E402
from kat_runner import HostBackend, run_kat  # noqa: E402


def P(a: np.ndarray):
    return C.c_void_p(a.ctypes.data)


def main() -> None:
    so = REPO / "oracle" / "_ref" / "libtrba_ref_omp.so"
    if not so.exists():
        raise SystemExit("build the reference first: make -C oracle ref")
    R = _typed_cpu_backend(so)
    check_formulas(R)
    out = run_kat(HostBackend(R))
    dst = REPO / "tests" / "golden" / "ref_kat.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


def check_formulas(R) -> None:
    """Assert the reference backend reproduces each unit test's own expected
    formula on these inputs (what the reference's cargo test checks)."""
    out: dict[str, np.ndarray] = {}

    # int8 GEMM (src/tests.rs:72-103): padded operands, compact s32 result
    for (m, n, k) in kat.GEMM_SHAPES:
        a, b, want = kat.gemm_case(m, n, k)
        ap, bp = kat.pad2(a, m, k), kat.pad2(b, n, k)
        c = np.zeros((m, n), dtype=np.int32)
        R.launch_gemm_int8(P(ap), P(bp), P(c), m, n, k, None)
        assert np.array_equal(c, want), (m, n, k)
        out[f"gemm_{m}_{n}_{k}"] = c

    # im2col (src/tests.rs:192-228)
    b, ch, h, w, k, s, p = kat.IM2COL_CASE
    inp = kat.det_i8(b * ch * h * w, 7)
    want, ho, wo = kat.ref_im2col(inp, b, ch, h, w, k, k, s, s, p, p)
    kp, rows = kat.a16(ch * k * k), b * ho * wo
    col = np.full((kat.a16(rows), kp), 0x55, dtype=np.int8)
    R.launch_im2col_pad(P(inp), P(col), b, ch, h, w, k, k, s, s, p, p, ho, wo, kp, None)
    assert np.array_equal(col[:rows, :ch * k * k], want)
    assert not col[:rows, ch * k * k:].any() and not col[rows:].any()
    out["im2col"] = col

    # conv epilogue (src/tests.rs:233-264)
    b, ch, ho, wo = kat.EPILOGUE_CASE
    acc = kat.det_i32(b * ho * wo * ch, 9, 3000.0)
    bias = kat.det(ch, 11)
    o = np.zeros(b * ch * ho * wo, dtype=np.int8)
    R.launch_conv_epilogue(P(acc), P(bias), P(o), ch, 127.0, 50.0, b, ch, ho, wo, None)
    assert np.array_equal(o, kat.conv_epilogue_ref(acc, bias, ch, b, ch, ho, wo))
    out["conv_epilogue"] = o

    dims = lambda s: (s["b"], s["cin"], s["h"], s["w"], s["cout"], s["kh"], s["kw"], s["sh"], s["sw"],
                      s["ph"], s["pw"], s["ho"], s["wo"])
    # fused backward grad_W (src/tests.rs:373-400)
    for i, s in enumerate(kat.GRAD_W_SHAPES):
        inp = kat.det_i8(s["b"] * s["cin"] * s["h"] * s["w"], 13)
        go = kat.det(s["b"] * s["cout"] * s["ho"] * s["wo"], 17)
        gw = np.zeros(s["cout"] * s["cin"] * s["kh"] * s["kw"], dtype=np.float32)
        R.launch_conv_backward_grad_weight(P(inp), P(go), P(gw), *dims(s), None)
        want = kat.ref_grad_w(s, inp, go)
        assert np.abs(gw - want).max() <= 1e-3 * max(1.0, np.abs(want).max())
        out[f"grad_w_{i}"] = gw

    # grad bias (src/tests.rs:402-432)
    s = kat.GRAD_BIAS_SHAPE
    go = kat.det(s["b"] * s["cout"] * s["ho"] * s["wo"], 19)
    gb = np.zeros(s["cout"], dtype=np.float32)
    R.launch_conv_backward_grad_bias(P(go), P(gb), s["b"], s["cout"], s["ho"], s["wo"], None)
    want = go.reshape(s["b"], s["cout"], -1).astype(np.float64).sum(axis=(0, 2))
    assert np.abs(gb - want).max() <= 1e-3 * max(1.0, np.abs(want).max())
    out["grad_bias"] = gb

    # grad input fp32 (src/tests.rs:434-459) and int8-weight (:572-636)
    for i, s in enumerate(kat.GRAD_IN_I8_SHAPES):
        go = kat.det(s["b"] * s["cout"] * s["ho"] * s["wo"], 23)
        cols = s["cin"] * s["kh"] * s["kw"]
        gi = np.zeros(s["b"] * s["cin"] * s["h"] * s["w"], dtype=np.float32)
        if i < len(kat.GRAD_IN_SHAPES):
            wt = kat.det(s["cout"] * cols, 29)
            R.launch_conv_backward_grad_input(P(go), P(wt), P(gi), *dims(s), None)
            want = kat.ref_grad_input(s, go, wt)
            assert np.abs(gi - want).max() <= 1e-3 * max(1.0, np.abs(want).max()) + 1e-3
            out[f"grad_input_{i}"] = gi.copy()
        raw = kat.det(s["cout"] * cols, 29)
        wq, ws = kat.host_requantize(raw)
        wpad = kat.pad2(wq, s["cout"], cols)
        R.launch_conv_backward_grad_input_i8(P(go), P(wpad), wpad.shape[1], float(ws), P(gi), *dims(s), None)
        want = kat.ref_grad_input(s, go, wq.astype(np.float32) * ws)
        assert np.abs(gi - want).max() <= 1e-4 * max(1.0, np.abs(want).max()) + 1e-4
        out[f"grad_input_i8_{i}"] = gi.copy()
        out[f"grad_input_i8_{i}_ws"] = np.array([ws], dtype=np.float32)

    # maxpool int8 forward/backward (src/tests.rs:473-532)
    for i, (b, ch, h, w, ties) in enumerate(kat.MAXPOOL_CASES):
        x = kat.maxpool_input(b, ch, h, w, ties)
        y = np.zeros(b * ch * (h // 2) * (w // 2), dtype=np.int8)
        go = kat.det(y.size, 53)
        dx = np.full(x.size, 777.0, dtype=np.float32)
        R.launch_maxpool2x2_forward_i8(P(x), P(y), b, ch, h, w, None)
        R.launch_maxpool2x2_backward_i8(P(x), P(go), P(dx), b, ch, h, w, None)
        want_y, idx = kat.maxpool_with_indices(x, b, ch, h, w)
        want_dx = np.zeros(x.size, dtype=np.float32)
        np.add.at(want_dx, idx, go)
        assert np.array_equal(y, want_y) and np.array_equal(dx, want_dx)
        out[f"maxpool_y_{i}"], out[f"maxpool_dx_{i}"] = y, dx

    # weight requantisation (src/tests.rs:640-690)
    for (rows, col) in kat.REQUANT_SHAPES:
        wv = kat.det(rows * col, 31) * np.float32(0.3)
        mx = np.zeros(1, dtype=np.float32)
        ws = np.zeros(1, dtype=np.float32)
        q = np.full((kat.a16(rows), kat.a16(col)), 0x55, dtype=np.int8)
        R.launch_max_abs_f32(P(wv), P(mx), wv.size, None)
        R.launch_quantize_pad_i8(P(wv), P(mx), P(ws), P(q), rows, col, kat.a16(col), None)
        hq, hws = kat.host_requantize(wv)
        assert ws[0] == hws and np.array_equal(q, kat.pad2(hq, rows, col))
        out[f"requant_{rows}_{col}"], out[f"requant_{rows}_{col}_ws"] = q, ws

    # device Adam (src/tests.rs:693-741)
    p, g, m, v = kat.adam_inputs()
    hp = kat.ADAM_HP
    P_, M_, V_ = p.copy(), m.copy(), v.copy()
    R.launch_adam_f32(P(P_), P(g), P(M_), P(V_), kat.ADAM_N, hp["lr"], hp["wd"], hp["clip"], hp["b1"],
                      hp["b2"], hp["eps"], hp["bc1"], hp["bc2"], None)
    wp, wm, wv = kat.adam_host(p, g, m, v, **hp)
    assert np.array_equal(P_, wp) and np.array_equal(M_, wm) and np.array_equal(V_, wv)
    out["adam_p"], out["adam_m"], out["adam_v"] = P_, M_, V_



if __name__ == "__main__":
    main()
