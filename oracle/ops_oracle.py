"""Test infrastructure only: CPU oracle of the reference's INT8 operator API
(LinearInt8 in src/linear.rs, LSTMInt8 / BiLSTMInt8 in src/bilstm.rs).

Plain numpy restatements, float32 where the reference computes in f32 with
the same operation order, used by tests/ to check libtrba_b200's operator
entry points (include/trba_ops.h).  Nothing in the product imports this file.

Arithmetic notes (Rust semantics):
  * `(x / s).clamp(-127, 127).round() as i8` rounds half away from zero;
  * `a * b + c` on f32 is two rounded operations (no FMA contraction);
  * `f32::exp` / `f32::tanh` come from the platform libm; here they are
    evaluated in f64 and rounded once (correctly rounded), which the tests
    allow for with the BiLSTM tolerance of the reference's tests (1e-4).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
ACC_DIVISOR = F32(127.0)       # src/conv2d.rs:24
ACTIVATION_SCALE = F32(10.0)   # src/bilstm.rs:29


def a16(x: int) -> int:
    return (x + 15) & ~15


def round_half_away(x: np.ndarray) -> np.ndarray:
    """Rust f32::round: half away from zero (f64 keeps |x| + 0.5 exact)."""
    x = np.asarray(x, F32).astype(np.float64)
    return (np.sign(x) * np.floor(np.abs(x) + 0.5)).astype(F32)


def quantize(w: np.ndarray) -> np.ndarray:
    """LinearInt8::quantize / LSTMInt8::quantize (src/linear.rs:53-59,
    src/bilstm.rs:57-63): per-tensor scale max|w|/127 (1.0 when all zero)."""
    w = np.asarray(w, F32)
    mx = F32(np.abs(w).max()) if w.size else F32(0.0)
    s = F32(mx / F32(127.0)) if mx > 0 else F32(1.0)
    q = np.clip((w / s).astype(F32), F32(-127.0), F32(127.0))
    return round_half_away(q).astype(np.int8)


def gemm_int8(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
    """C s32 [m, n] = A [m, k] . B [n, k]^T (launch_gemm_int8 contract)."""
    A = np.asarray(a, np.int8).reshape(m, k).astype(np.int64)
    B = np.asarray(b, np.int8).reshape(n, k).astype(np.int64)
    return (A @ B.T).astype(np.int32)


class LinearInt8:
    """src/linear.rs:12-180."""

    def __init__(self, weight_f32: np.ndarray, bias: np.ndarray, in_features: int, out_features: int):
        self.in_features, self.out_features = in_features, out_features
        self.weight_f32 = np.asarray(weight_f32, F32).reshape(out_features * in_features).copy()
        self.bias = np.asarray(bias, F32).reshape(out_features).copy()
        self.grad_f32 = np.zeros_like(self.weight_f32)
        self.requantize()

    def requantize(self):
        self.weight_int8 = quantize(self.weight_f32)

    def forward(self, inp: np.ndarray) -> np.ndarray:
        """src/linear.rs:66-115: [rows, in] int8 -> [rows, out] int32."""
        inp = np.asarray(inp, np.int8).ravel()
        assert inp.size and inp.size % self.in_features == 0
        rows = inp.size // self.in_features
        return gemm_int8(inp, self.weight_int8, rows, self.out_features, self.in_features).ravel()

    def backward(self, inp: np.ndarray, grad_out: np.ndarray, lr: float, mom: float) -> float:
        """src/linear.rs:121-175: batch-averaged f32 outer product, global-norm
        clip at 10, SGD, non-finite -> 0, re-quantise.  Returns the clip factor."""
        fi, fo = self.in_features, self.out_features
        inp = np.asarray(inp, F32).ravel()
        go = np.asarray(grad_out, F32).ravel()
        rows = inp.size // fi if fi > 0 else 0
        if rows == 0 or go.size < rows * fo:
            return 0.0
        inv_rows = F32(1.0) / F32(rows)
        X = inp[:rows * fi].reshape(rows, fi)
        G = go[:rows * fo].reshape(rows, fo)
        acc = np.zeros((fo, fi), F32)
        for r in range(rows):  # sequential f32 accumulation over rows, as the reference
            acc = (acc + (G[r][:, None] * X[r][None, :]).astype(F32)).astype(F32)
        grad = (acc * inv_rows).astype(F32)
        self.grad_f32 = grad.ravel()
        # f32 squares summed in f64 and rounded once (the reference sums the
        # f32 squares in a rayon tree whose order is not fixed)
        norm = F32(np.sqrt(F32(np.sum((grad * grad).astype(F32).astype(np.float64)))))
        clip = F32(F32(10.0) / norm) if norm > F32(10.0) else F32(1.0)
        step = F32(F32(lr) * clip)
        w = (self.weight_f32 - (step * self.grad_f32).astype(F32)).astype(F32)
        self.weight_f32 = np.where(np.isfinite(w), w, F32(0.0)).astype(F32)
        gb = np.zeros(fo, F32)
        for r in range(rows):
            gb = (gb + G[r]).astype(F32)
        b = (self.bias - ((step * gb).astype(F32) * inv_rows).astype(F32)).astype(F32)
        self.bias = np.where(np.isfinite(b), b, F32(0.0)).astype(F32)
        self.requantize()
        return float(clip)


def _exp32(x):
    # exp beyond the f32 range rounds to inf, as f32::exp overflows
    with np.errstate(over="ignore"):
        return np.exp(np.asarray(x, F32).astype(np.float64)).astype(F32)


def _tanh32(x):
    return np.tanh(np.asarray(x, F32).astype(np.float64)).astype(F32)


def sigmoid32(x):
    """src/bilstm.rs:258-261: 1 / (1 + exp(-x)) in f32."""
    e = _exp32(-np.asarray(x, F32))
    return (F32(1.0) / (F32(1.0) + e).astype(F32)).astype(F32)


class LSTMInt8:
    """src/bilstm.rs:13-178."""

    def __init__(self, w_ih, w_hh, bias, input_size: int, hidden_size: int):
        self.input_size, self.hidden_size = input_size, hidden_size
        self.weight_ih_f32 = np.asarray(w_ih, F32).ravel().copy()
        self.weight_hh_f32 = np.asarray(w_hh, F32).ravel().copy()
        self.bias = np.asarray(bias, F32).ravel().copy()
        self.requantize()

    def requantize(self):
        self.weight_ih_int8 = quantize(self.weight_ih_f32)
        self.weight_hh_int8 = quantize(self.weight_hh_f32)

    @staticmethod
    def quantize_h(h: np.ndarray) -> np.ndarray:
        """src/bilstm.rs:84-87: round(clamp(h * 10, +-127)) as i8."""
        v = np.clip((np.asarray(h, F32) * ACTIVATION_SCALE).astype(F32), F32(-127.0), F32(127.0))
        return round_half_away(v).astype(np.int8)

    def i2h_forward(self, x_int8, batch):
        return gemm_int8(x_int8, self.weight_ih_int8, batch, 4 * self.hidden_size, self.input_size).ravel()

    def h2h_forward(self, h_int8, batch):
        return gemm_int8(h_int8, self.weight_hh_int8, batch, 4 * self.hidden_size, self.hidden_size).ravel()

    def forward_step(self, x_int8, h_prev, c_prev, batch):
        """src/bilstm.rs:72-117 -> (h_new, c_new), each [batch, hidden] f32."""
        hs = self.hidden_size
        gi = self.i2h_forward(x_int8, batch).reshape(batch, 4 * hs)
        gh = self.h2h_forward(self.quantize_h(h_prev), batch).reshape(batch, 4 * hs)
        inv = F32(F32(1.0) / (ACC_DIVISOR * ACTIVATION_SCALE))
        pre = ((gi.astype(F32) + gh.astype(F32)).astype(F32) * inv).astype(F32)
        pre = (pre + self.bias[None, :]).astype(F32)
        ig = sigmoid32(pre[:, 0:hs])
        fg = sigmoid32(pre[:, hs:2 * hs])
        cg = _tanh32(pre[:, 2 * hs:3 * hs])
        og = sigmoid32(pre[:, 3 * hs:4 * hs])
        cp = np.asarray(c_prev, F32).reshape(batch, hs)
        c = ((fg * cp).astype(F32) + (ig * cg).astype(F32)).astype(F32)
        h = (og * _tanh32(c)).astype(F32)
        return h.ravel(), c.ravel()


class BiLSTMInt8:
    """src/bilstm.rs:180-256.  Both directions step through time in the same
    (forward) order, as the reference does; the output is each direction's
    hidden state averaged over time, [batch, 2*hidden]."""

    def __init__(self, fwd: LSTMInt8, bwd: LSTMInt8):
        self.forward_lstm, self.backward_lstm = fwd, bwd
        self.hidden_size = fwd.hidden_size

    def forward(self, x_seq_int8, batch, seq_len):
        inp, hs = self.forward_lstm.input_size, self.hidden_size
        x = np.asarray(x_seq_int8, np.int8).ravel()
        assert x.size >= seq_len * batch * inp

        def run(lstm):
            h = np.zeros(batch * hs, F32)
            c = np.zeros(batch * hs, F32)
            out = []
            for t in range(seq_len):
                h, c = lstm.forward_step(x[t * batch * inp:(t + 1) * batch * inp], h, c, batch)
                out.append(h)
            return out

        f, b = run(self.forward_lstm), run(self.backward_lstm)
        inv_t = F32(F32(1.0) / F32(max(seq_len, 1)))
        sf = np.zeros(batch * hs, F32)
        sb = np.zeros(batch * hs, F32)
        for t in range(seq_len):
            sf = (sf + f[t]).astype(F32)
            sb = (sb + b[t]).astype(F32)
        out = np.empty((batch, 2 * hs), F32)
        out[:, :hs] = (sf * inv_t).astype(F32).reshape(batch, hs)
        out[:, hs:] = (sb * inv_t).astype(F32).reshape(batch, hs)
        return out.ravel()
