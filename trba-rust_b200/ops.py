"""Python mirror of the reference's INT8 operator API over libtrba_b200
(include/trba_ops.h): LinearInt8 (src/linear.rs), LSTMInt8 and BiLSTMInt8
(src/bilstm.rs).  Method names, argument meaning and return values follow
the Rust structs; weights are injected (the reference draws them from
rand::thread_rng), and all state lives on the device.

    lin = LinearInt8(in_features, out_features, weight_f32, bias)
    out = lin.forward(inp_int8)                   # [rows*out] int32
    clip = lin.backward(inp_f32, grad_out, lr, mom)
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .ffi import lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return C.c_void_p(a.ctypes.data)


def _err(L, what):
    return RuntimeError(f"{what}: " + L.trba_last_error_string().decode())


class LinearInt8:
    """src/linear.rs:12-180."""

    def __init__(self, in_features: int, out_features: int, weight_f32: np.ndarray, bias: np.ndarray | None = None):
        self.L = lib()
        self.in_features, self.out_features = in_features, out_features
        w = np.ascontiguousarray(weight_f32, np.float32).reshape(out_features * in_features)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32).reshape(out_features)
        self.h = self.L.trba_linear_int8_create(in_features, out_features, _p(w), None if b is None else _p(b))
        if not self.h:
            raise _err(self.L, "LinearInt8::new")

    def close(self):
        if getattr(self, "h", None):
            self.L.trba_linear_int8_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _state(self):
        n = self.in_features * self.out_features
        w, q = np.empty(n, np.float32), np.empty(n, np.int8)
        b, g = np.empty(self.out_features, np.float32), np.empty(n, np.float32)
        if self.L.trba_linear_int8_get(self.h, _p(w), _p(q), _p(b), _p(g)) != 0:
            raise _err(self.L, "LinearInt8 state")
        return w, q, b, g

    @property
    def weight_f32(self) -> np.ndarray:
        return self._state()[0]

    @weight_f32.setter
    def weight_f32(self, w):
        w = np.ascontiguousarray(w, np.float32).reshape(-1)
        if self.L.trba_linear_int8_set(self.h, _p(w), None) != 0:
            raise _err(self.L, "LinearInt8 set weights")

    @property
    def weight_int8(self) -> np.ndarray:
        return self._state()[1]

    @property
    def bias(self) -> np.ndarray:
        return self._state()[2]

    @property
    def grad_f32(self) -> np.ndarray:
        return self._state()[3]

    def requantize(self):
        self.L.trba_linear_int8_requantize(self.h, None)

    def forward(self, inp: np.ndarray) -> np.ndarray:
        """[rows, in] int8 -> [rows*out] int32 (src/linear.rs:66-115)."""
        inp = np.ascontiguousarray(inp, np.int8).reshape(-1)
        if inp.size == 0 or inp.size % self.in_features:
            raise ValueError(f"LinearInt8::forward: input {inp.size} is not a multiple of in_features "
                             f"{self.in_features}")
        out = np.empty(inp.size // self.in_features * self.out_features, np.int32)
        if self.L.trba_linear_int8_forward_host(self.h, _p(inp), inp.size, _p(out)) != 0:
            raise _err(self.L, "LinearInt8::forward")
        return out

    def backward(self, inp: np.ndarray, grad_out: np.ndarray, lr: float, mom: float) -> float:
        """FP32 backward + SGD with global-norm clipping; returns the clip
        factor (src/linear.rs:121-175)."""
        inp = np.ascontiguousarray(inp, np.float32).reshape(-1)
        go = np.ascontiguousarray(grad_out, np.float32).reshape(-1)
        return float(self.L.trba_linear_int8_backward_host(self.h, _p(inp), inp.size, _p(go), go.size,
                                                           float(lr), float(mom)))

    def param_count(self) -> int:
        return int(self.L.trba_linear_int8_param_count(self.h))


class LSTMInt8:
    """src/bilstm.rs:13-178.  forward_step etc. take host numpy arrays."""

    def __init__(self, input_size: int, hidden_size: int, w_ih: np.ndarray, w_hh: np.ndarray,
                 bias: np.ndarray | None = None):
        self.L = lib()
        self.input_size, self.hidden_size = input_size, hidden_size
        wi = np.ascontiguousarray(w_ih, np.float32).reshape(-1)
        wh = np.ascontiguousarray(w_hh, np.float32).reshape(-1)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32).reshape(-1)
        self.h = self.L.trba_lstm_int8_create(input_size, hidden_size, _p(wi), _p(wh), None if b is None else _p(b))
        if not self.h:
            raise _err(self.L, "LSTMInt8::new")

    def close(self):
        if getattr(self, "h", None):
            self.L.trba_lstm_int8_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def state(self):
        G, I, H = 4 * self.hidden_size, self.input_size, self.hidden_size
        wi, qi = np.empty(G * I, np.float32), np.empty(G * I, np.int8)
        wh, qh = np.empty(G * H, np.float32), np.empty(G * H, np.int8)
        b = np.empty(G, np.float32)
        if self.L.trba_lstm_int8_get(self.h, _p(wi), _p(qi), _p(wh), _p(qh), _p(b)) != 0:
            raise _err(self.L, "LSTMInt8 state")
        return {"weight_ih_f32": wi, "weight_ih_int8": qi, "weight_hh_f32": wh, "weight_hh_int8": qh, "bias": b}

    def requantize(self):
        self.L.trba_lstm_int8_requantize(self.h, None)

    def forward_step(self, x_int8, h_prev, c_prev, batch_size: int):
        """src/bilstm.rs:72-117 -> (h_new, c_new) as float32 [batch*hidden]."""
        import torch
        x = torch.from_numpy(np.ascontiguousarray(x_int8, np.int8).reshape(-1)).cuda()
        hp = torch.from_numpy(np.ascontiguousarray(h_prev, np.float32).reshape(-1)).cuda()
        cp = torch.from_numpy(np.ascontiguousarray(c_prev, np.float32).reshape(-1)).cuda()
        hn = torch.empty(batch_size * self.hidden_size, dtype=torch.float32, device="cuda")
        cn = torch.empty_like(hn)
        rc = self.L.trba_lstm_int8_forward_step(self.h, C.c_void_p(x.data_ptr()), C.c_void_p(hp.data_ptr()),
                                                C.c_void_p(cp.data_ptr()), batch_size, C.c_void_p(hn.data_ptr()),
                                                C.c_void_p(cn.data_ptr()), None)
        if rc != 0:
            raise _err(self.L, "LSTMInt8::forward_step")
        return hn.cpu().numpy(), cn.cpu().numpy()

    def _proj(self, fn, a, batch, k):
        import torch
        t = torch.from_numpy(np.ascontiguousarray(a, np.int8).reshape(-1)).cuda()
        out = torch.empty(batch * 4 * self.hidden_size, dtype=torch.int32, device="cuda")
        if fn(self.h, C.c_void_p(t.data_ptr()), batch, C.c_void_p(out.data_ptr()), None) != 0:
            raise _err(self.L, "LSTMInt8 projection")
        return out.cpu().numpy()

    def i2h_forward(self, x_int8, batch: int):
        return self._proj(self.L.trba_lstm_int8_i2h_forward, x_int8, batch, self.input_size)

    def h2h_forward(self, h_int8, batch: int):
        return self._proj(self.L.trba_lstm_int8_h2h_forward, h_int8, batch, self.hidden_size)

    @staticmethod
    def gemm_int8(a, b, m: int, n: int, k: int) -> np.ndarray:
        """src/bilstm.rs:132-173 on compact operands."""
        import torch
        L = lib()
        ta = torch.from_numpy(np.ascontiguousarray(a, np.int8).reshape(-1)).cuda()
        tb = torch.from_numpy(np.ascontiguousarray(b, np.int8).reshape(-1)).cuda()
        out = torch.empty(m * n, dtype=torch.int32, device="cuda")
        if L.trba_gemm_int8_compact(C.c_void_p(ta.data_ptr()), C.c_void_p(tb.data_ptr()),
                                    C.c_void_p(out.data_ptr()), m, n, k, None) != 0:
            raise _err(L, "LSTMInt8::gemm_int8")
        return out.cpu().numpy()

    def param_count(self) -> int:
        return int(self.L.trba_lstm_int8_param_count(self.h))


class BiLSTMInt8:
    """src/bilstm.rs:180-256."""

    def __init__(self, forward: LSTMInt8, backward: LSTMInt8):
        self.forward_lstm, self.backward_lstm = forward, backward
        self.hidden_size = forward.hidden_size

    def forward(self, x_seq_int8, batch_size: int, seq_len: int) -> np.ndarray:
        """x [seq_len, batch, input] int8 -> [batch * 2*hidden] float32."""
        import torch
        L = lib()
        need = seq_len * batch_size * self.forward_lstm.input_size
        x = np.ascontiguousarray(x_seq_int8, np.int8).reshape(-1)
        if x.size < need:
            raise ValueError(f"BiLSTM::forward: input is {x.size} bytes, need {need}")
        t = torch.from_numpy(x[:max(need, 1)].copy()).cuda()
        out = torch.empty(batch_size * 2 * self.hidden_size, dtype=torch.float32, device="cuda")
        if L.trba_bilstm_int8_forward(self.forward_lstm.h, self.backward_lstm.h, C.c_void_p(t.data_ptr()),
                                      batch_size, seq_len, C.c_void_p(out.data_ptr()), None) != 0:
            raise _err(L, "BiLSTMInt8::forward")
        return out.cpu().numpy()

    def param_count(self) -> int:
        return self.forward_lstm.param_count() + self.backward_lstm.param_count()
