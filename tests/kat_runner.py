"""Runs the reference unit tests' known-answer cases (tests/kat.py) through
any implementation of the reference's backend ABI:

  HostBackend  — a CPU library whose "device" pointers are host pointers
                 (the oracle, or the reference's own CPU backend);
  CudaBackend  — libtrba_b200.so, with device buffers from torch (plumbing).

Both return the same dict of numpy outputs, compared against
tests/golden/ref_kat.npz by the tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

import kat


class HostBackend:
    def __init__(self, L):
        self.L = L

    def buf(self, a: np.ndarray):
        return np.ascontiguousarray(a).copy()

    def ptr(self, h):
        return C.c_void_p(h.ctypes.data)

    def get(self, h) -> np.ndarray:
        return h.copy()

    stream = None

    def sync(self):
        pass


class CudaBackend:
    def __init__(self, L):
        import torch
        self.L, self.torch = L, torch
        self.stream = None  # legacy default stream: ordered with torch's default stream

    def buf(self, a: np.ndarray):
        t = self.torch.from_numpy(np.ascontiguousarray(a).copy())
        return t.to("cuda")

    def ptr(self, h):
        return C.c_void_p(h.data_ptr())

    def get(self, h) -> np.ndarray:
        self.torch.cuda.synchronize()
        return h.cpu().numpy().copy()

    def sync(self):
        self.torch.cuda.synchronize()


def run_kat(be) -> dict[str, np.ndarray]:
    L, P, out = be.L, be.ptr, {}
    st = be.stream

    for (m, n, k) in kat.GEMM_SHAPES:
        a, b, _ = kat.gemm_case(m, n, k)
        A, B = be.buf(kat.pad2(a, m, k)), be.buf(kat.pad2(b, n, k))
        Cc = be.buf(np.full((m, n), -7, dtype=np.int32))
        L.launch_gemm_int8(P(A), P(B), P(Cc), m, n, k, st)
        out[f"gemm_{m}_{n}_{k}"] = be.get(Cc)

    b, ch, h, w, k, s, p = kat.IM2COL_CASE
    ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    kp, rows = kat.a16(ch * k * k), b * ho * wo
    X = be.buf(kat.det_i8(b * ch * h * w, 7))
    COL = be.buf(np.full((kat.a16(rows), kp), 0x55, dtype=np.int8))
    L.launch_im2col_pad(P(X), P(COL), b, ch, h, w, k, k, s, s, p, p, ho, wo, kp, st)
    out["im2col"] = be.get(COL)

    b, ch, ho, wo = kat.EPILOGUE_CASE
    ACC = be.buf(kat.det_i32(b * ho * wo * ch, 9, 3000.0))
    BIAS = be.buf(kat.det(ch, 11))
    O = be.buf(np.zeros(b * ch * ho * wo, dtype=np.int8))
    L.launch_conv_epilogue(P(ACC), P(BIAS), P(O), ch, 127.0, 50.0, b, ch, ho, wo, st)
    out["conv_epilogue"] = be.get(O)

    def dims(s):
        return (s["b"], s["cin"], s["h"], s["w"], s["cout"], s["kh"], s["kw"], s["sh"], s["sw"],
                s["ph"], s["pw"], s["ho"], s["wo"])

    for i, s in enumerate(kat.GRAD_W_SHAPES):
        IN = be.buf(kat.det_i8(s["b"] * s["cin"] * s["h"] * s["w"], 13))
        GO = be.buf(kat.det(s["b"] * s["cout"] * s["ho"] * s["wo"], 17))
        GW = be.buf(np.zeros(s["cout"] * s["cin"] * s["kh"] * s["kw"], dtype=np.float32))
        L.launch_conv_backward_grad_weight(P(IN), P(GO), P(GW), *dims(s), st)
        out[f"grad_w_{i}"] = be.get(GW)

    s = kat.GRAD_BIAS_SHAPE
    GO = be.buf(kat.det(s["b"] * s["cout"] * s["ho"] * s["wo"], 19))
    GB = be.buf(np.zeros(s["cout"], dtype=np.float32))
    L.launch_conv_backward_grad_bias(P(GO), P(GB), s["b"], s["cout"], s["ho"], s["wo"], st)
    out["grad_bias"] = be.get(GB)

    for i, s in enumerate(kat.GRAD_IN_I8_SHAPES):
        GO = be.buf(kat.det(s["b"] * s["cout"] * s["ho"] * s["wo"], 23))
        cols = s["cin"] * s["kh"] * s["kw"]
        n_in = s["b"] * s["cin"] * s["h"] * s["w"]
        if i < len(kat.GRAD_IN_SHAPES):
            WT = be.buf(kat.det(s["cout"] * cols, 29))
            GI = be.buf(np.zeros(n_in, dtype=np.float32))
            L.launch_conv_backward_grad_input(P(GO), P(WT), P(GI), *dims(s), st)
            out[f"grad_input_{i}"] = be.get(GI)
        wq, ws = kat.host_requantize(kat.det(s["cout"] * cols, 29))
        wpad = kat.pad2(wq, s["cout"], cols)
        WQ = be.buf(wpad)
        GI = be.buf(np.zeros(n_in, dtype=np.float32))
        L.launch_conv_backward_grad_input_i8(P(GO), P(WQ), wpad.shape[1], float(ws), P(GI), *dims(s), st)
        out[f"grad_input_i8_{i}"] = be.get(GI)
        out[f"grad_input_i8_{i}_ws"] = np.array([ws], dtype=np.float32)

    for i, (b, ch, h, w, ties) in enumerate(kat.MAXPOOL_CASES):
        x = kat.maxpool_input(b, ch, h, w, ties)
        ny = b * ch * (h // 2) * (w // 2)
        X, Y = be.buf(x), be.buf(np.zeros(ny, dtype=np.int8))
        GO = be.buf(kat.det(ny, 53))
        DX = be.buf(np.full(x.size, 777.0, dtype=np.float32))
        L.launch_maxpool2x2_forward_i8(P(X), P(Y), b, ch, h, w, st)
        L.launch_maxpool2x2_backward_i8(P(X), P(GO), P(DX), b, ch, h, w, st)
        out[f"maxpool_y_{i}"], out[f"maxpool_dx_{i}"] = be.get(Y), be.get(DX)

    for (rows, col) in kat.REQUANT_SHAPES:
        W = be.buf(kat.det(rows * col, 31) * np.float32(0.3))
        MX, WS = be.buf(np.zeros(1, np.float32)), be.buf(np.zeros(1, np.float32))
        Q = be.buf(np.full((kat.a16(rows), kat.a16(col)), 0x55, dtype=np.int8))
        L.launch_max_abs_f32(P(W), P(MX), rows * col, st)
        L.launch_quantize_pad_i8(P(W), P(MX), P(WS), P(Q), rows, col, kat.a16(col), st)
        out[f"requant_{rows}_{col}"], out[f"requant_{rows}_{col}_ws"] = be.get(Q), be.get(WS)

    p, g, m, v = kat.adam_inputs()
    hp = kat.ADAM_HP
    PP, G, M, V = be.buf(p), be.buf(g), be.buf(m), be.buf(v)
    L.launch_adam_f32(P(PP), P(G), P(M), P(V), kat.ADAM_N, hp["lr"], hp["wd"], hp["clip"], hp["b1"],
                      hp["b2"], hp["eps"], hp["bc1"], hp["bc2"], st)
    out["adam_p"], out["adam_m"], out["adam_v"] = be.get(PP), be.get(M), be.get(V)
    return out


# Tolerance per output: exact for the integer / quantisation path and for
# Adam (f64 arithmetic restated op for op); the reference tests' own
# tolerances for the fp32 gathers.
def tolerance(key: str):
    if key.startswith("grad_w_") or key == "grad_bias" or (key.startswith("grad_input_") and "i8" not in key):
        return "rel1e-3"
    if key.startswith("grad_input_i8_") and not key.endswith("_ws"):
        return "rel1e-4"
    return "exact"


def compare(got: dict, want: dict) -> list[str]:
    bad = []
    for k, w in want.items():
        if k not in got:
            bad.append(f"{k}: missing")
            continue
        g = got[k]
        tol = tolerance(k)
        if tol == "exact":
            if g.shape != w.shape or not np.array_equal(g, w):
                nd = int((g != w).sum()) if g.shape == w.shape else -1
                bad.append(f"{k}: {nd} elements differ")
        else:
            r = 1e-3 if tol == "rel1e-3" else 1e-4
            d = float(np.abs(g.astype(np.float64) - w).max())
            lim = r * max(1.0, float(np.abs(w).max())) + r
            if not d <= lim:
                bad.append(f"{k}: max diff {d} > {lim}")
    return bad
