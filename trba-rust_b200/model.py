"""Python binding of the fused QAT training step (include/trba_qat.h).

    m = QatModel(Config(batch=48))          # allocates every buffer once
    m.set_params(flat_fp32)                 # manifest order, host numpy
    loss = m.train_step_host(img, text_in, target, ctc_tgt, ctc_len)

The heavy lifting is libtrba_b200.so; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields

import numpy as np

from .ffi import lib


class _Cfg(C.Structure):
    _fields_ = [("fd", C.c_int), ("hidden", C.c_int), ("classes", C.c_int), ("img_h", C.c_int),
                ("img_w", C.c_int), ("max_len", C.c_int), ("rnn_layers", C.c_int), ("batch", C.c_int),
                ("sos", C.c_int), ("eos", C.c_int), ("pad", C.c_int), ("lr", C.c_float),
                ("weight_decay", C.c_float), ("ctc_weight", C.c_float), ("muon_cap", C.c_float),
                ("clip_warmup", C.c_int), ("wgrad_mode", C.c_int), ("dgrad_mode", C.c_int),
                ("wq_per_channel", C.c_int), ("inference_only", C.c_int), ("conv_fwd_mode", C.c_int)]


@dataclass
class Config:
    fd: int = 128
    hidden: int = 64
    classes: int = 130
    img_h: int = 32
    img_w: int = 160
    max_len: int = 20
    rnn_layers: int = 2
    batch: int = 48
    sos: int = 1
    eos: int = 2
    pad: int = 0
    lr: float = 5.107e-4
    weight_decay: float = 1.9548e-5
    ctc_weight: float = 0.03
    muon_cap: float = 10.0
    clip_warmup: int = 500
    wgrad_mode: int = 0  # 0: the reference's operand order, 1: dW = dX^T col
    dgrad_mode: int = 0  # conv input gradient: 0 exact f32 order, 1 tensor cores (bf16 x3 split)
    wq_per_channel: int = 0  # conv weight scales: 0 per tensor (the reference), 1 per output channel
    inference_only: int = 0  # 1: forward buffers only (serving); training calls are refused
    conv_fwd_mode: int = 1  # conv forward GEMM: 0 im2col + GEMM, 1 implicit GEMM (same accumulators)

    def to_c(self) -> _Cfg:
        return _Cfg(**{f.name: getattr(self, f.name) for f in fields(self)})

    @property
    def steps(self) -> int:
        return self.max_len + 1


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags.c_contiguous
        return C.c_void_p(a.ctypes.data)
    return C.c_void_p(a.data_ptr())  # torch tensor


class QatModel:
    def __init__(self, cfg: Config):
        self.cfg = cfg
        self.L = lib()
        self._c = cfg.to_c()
        self.h = self.L.trba_model_create(C.byref(self._c))
        if not self.h:
            raise RuntimeError("trba_model_create failed: " + self.L.trba_last_error_string().decode())
        self.n_params = int(self.L.trba_model_param_count(self.h))

    def close(self):
        if getattr(self, "h", None):
            self.L.trba_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def manifest(self):
        out = []
        name = C.create_string_buffer(128)
        off, rows, cols, kind = C.c_longlong(), C.c_int(), C.c_int(), C.c_int()
        for i in range(self.L.trba_model_param_entries(self.h)):
            self.L.trba_model_param_entry(self.h, i, name, 128, C.byref(off), C.byref(rows), C.byref(cols),
                                          C.byref(kind))
            out.append((name.value.decode(), off.value, rows.value, cols.value, kind.value))
        return out

    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed ({rc}): " + self.L.trba_last_error_string().decode())

    def set_params(self, flat: np.ndarray):
        flat = np.ascontiguousarray(flat, dtype=np.float32)
        self._check(self.L.trba_model_set_params(self.h, _ptr(flat), flat.size), "set_params")

    def get_params(self) -> np.ndarray:
        out = np.empty(self.n_params, np.float32)
        self._check(self.L.trba_model_get_params(self.h, _ptr(out), out.size), "get_params")
        return out

    def get_grads(self) -> np.ndarray:
        out = np.empty(self.n_params, np.float32)
        self._check(self.L.trba_model_get_grads(self.h, _ptr(out), out.size), "get_grads")
        return out

    def running_stats(self) -> np.ndarray:
        n = int(self.L.trba_model_running_stats_count(self.h))
        out = np.empty(n, np.float32)
        self._check(self.L.trba_model_get_running_stats(self.h, _ptr(out), n), "running_stats")
        return out

    def get_moments(self, m_out: np.ndarray, v_out: np.ndarray):
        """Adam first / second moments of every parameter (manifest order)."""
        self._check(self.L.trba_model_get_moments(self.h, _ptr(m_out), _ptr(v_out), self.n_params), "get_moments")

    def set_moments(self, m_in: np.ndarray, v_in: np.ndarray):
        m_in = np.ascontiguousarray(m_in, np.float32)
        v_in = np.ascontiguousarray(v_in, np.float32)
        self._check(self.L.trba_model_set_moments(self.h, _ptr(m_in), _ptr(v_in), self.n_params), "set_moments")

    def set_running_stats(self, rs: np.ndarray):
        rs = np.ascontiguousarray(rs, np.float32)
        self._check(self.L.trba_model_set_running_stats(self.h, _ptr(rs), rs.size), "set_running_stats")

    def step_count(self) -> int:
        return int(self.L.trba_model_step_count(self.h))

    def set_step_count(self, t: int):
        self._check(self.L.trba_model_set_step_count(self.h, int(t)), "set_step_count")

    def conv_channels(self) -> list:
        """Output channels of every convolution, in the running-statistics order."""
        return [rows for name, _, rows, cols, kind in self.manifest() if name.endswith(".gamma")]

    def debug_tensor(self, name: str, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self._check(self.L.trba_model_debug_tensor(self.h, name.encode(), _ptr(out), n), f"debug_tensor({name})")
        return out

    def forward_backward(self, img, text_in, target, ctc_tgt, ctc_len, stream=None):
        b = int(img.shape[0])
        self._check(self.L.trba_model_forward_backward(self.h, _ptr(img), _ptr(text_in), _ptr(target), _ptr(ctc_tgt),
                                                       _ptr(ctc_len), b, stream), "forward_backward")

    def optimizer_step(self, stream=None):
        self._check(self.L.trba_model_optimizer_step(self.h, stream), "optimizer_step")

    def train_step(self, img, text_in, target, ctc_tgt, ctc_len, stream=None):
        """Device inputs (torch CUDA tensors); returns nothing (loss stays on device)."""
        b = int(img.shape[0])
        self._check(self.L.trba_model_train_step(self.h, _ptr(img), _ptr(text_in), _ptr(target), _ptr(ctc_tgt),
                                                 _ptr(ctc_len), b, stream), "train_step")

    def train_step_host(self, img, text_in, target, ctc_tgt, ctc_len, stream=None) -> np.ndarray:
        """Host inputs (numpy, ideally pinned); returns [total, attn CE, CTC]."""
        b = int(img.shape[0])
        loss = np.zeros(3, np.float32)
        self._check(self.L.trba_model_train_step_host(self.h, _ptr(img), _ptr(text_in), _ptr(target), _ptr(ctc_tgt),
                                                      _ptr(ctc_len), b, _ptr(loss), stream), "train_step_host")
        return loss

    def infer(self, img, stream=None):
        """Greedy decoding of device images [B, 3, H, W] int8; returns the
        argmax token of every step, [max_len+1, B] int32 (synchronises)."""
        b = int(img.shape[0])
        self._check(self.L.trba_model_infer(self.h, _ptr(img), b, None, stream), "infer")
        out = np.empty((self.cfg.steps, b), np.int32)
        self.L.cuda_sync(None)
        self.L.cuda_memcpy_d2h(_ptr(out), self._step_tokens_ptr(), out.nbytes, None)
        return out

    def _step_tokens_ptr(self):
        return C.c_void_p(self.L.trba_model_step_tokens_dev(self.h))

    def infer_host(self, img, stream=None) -> list:
        """Greedy decoding of host images; the reference's output: one token
        list per line (eos not emitted, batch-level stop)."""
        img = np.ascontiguousarray(img, np.int8)
        b = int(img.shape[0])
        tok = np.empty((b, self.cfg.steps), np.int32)
        lens = np.empty(b, np.int32)
        self._check(self.L.trba_model_infer_host(self.h, _ptr(img), b, _ptr(tok), _ptr(lens), stream), "infer_host")
        return [tok[i, :lens[i]].tolist() for i in range(b)]

    def loss(self) -> np.ndarray:
        """[total, attention CE, CTC] of the last step (synchronises)."""
        out = np.zeros(3, np.float32)
        self.L.cuda_sync(None)
        self.L.cuda_memcpy_d2h(_ptr(out), self.L.trba_model_loss_dev(self.h), 12, None)
        return out

    def loss_dev_ptr(self) -> int:
        return C.cast(self.L.trba_model_loss_dev(self.h), C.c_void_p).value

    PROBE_CONV_GEMM, PROBE_WGRAD_GEMM, PROBE_DGRAD, PROBE_SGEMM = 0, 1, 2, 3
    PROBE_PHASES = {"cnn_forward": 4, "head_forward": 5, "head_backward": 6, "cnn_backward": 7,
                    "allreduce_optimizer": 8}

    def probe(self, kind: int):
        """Bracket every launch of one kernel family with CUDA events (-1 = off)."""
        self._check(self.L.trba_model_probe(self.h, kind), "probe")

    def probe_read(self):
        """(device ms summed over the probed launches, launches, algorithmic ops,
        algorithmic bytes, steps covered)."""
        ms, n, ops, nbytes, steps = C.c_double(), C.c_longlong(), C.c_double(), C.c_double(), C.c_longlong()
        self._check(self.L.trba_model_probe_read(self.h, C.byref(ms), C.byref(n), C.byref(ops), C.byref(nbytes),
                                                 C.byref(steps)), "probe_read")
        return ms.value, n.value, ops.value, nbytes.value, steps.value

    def use_graphs(self, enable: bool = True):
        """Record the step as a CUDA graph and replay it (inputs refreshed in place)."""
        self._check(self.L.trba_model_use_graphs(self.h, 1 if enable else 0), "use_graphs")

    def dp_init(self, id128: bytes, rank: int, world: int):
        buf = C.create_string_buffer(id128, 128)
        self._check(self.L.trba_dp_init(self.h, buf, rank, world), "dp_init")

    def dp_finalize(self):
        self.L.trba_dp_finalize(self.h)

    def dp_wait(self, stream=None, timeout_s: float = 60.0) -> int:
        """Wait for the queued step(s) on `stream`; a peer's NCCL failure or
        a step that does not finish within timeout_s aborts the communicator
        (trba_dp_wait).  Returns 0 (finished), 1 (NCCL error) or 2 (timeout)."""
        rc = self.L.trba_dp_wait(self.h, stream, float(timeout_s) * 1000.0)
        if rc < 0:
            raise RuntimeError("trba_dp_wait: " + self.L.trba_last_error_string().decode())
        return rc

    @staticmethod
    def dp_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        rc = lib().trba_dp_unique_id(buf)
        if rc != 0:
            raise RuntimeError(f"ncclGetUniqueId failed ({rc})")
        return buf.raw


def pack_labels(text_in, target, ctc_targets, steps):
    """int32 arrays for the C API: text_in/target [B, steps], ctc [B, steps]
    padded with -1, ctc lengths [B] (tokens plus eos)."""
    b = len(ctc_targets)
    ctc = np.full((b, steps), -1, np.int32)
    lens = np.zeros(b, np.int32)
    for i, t in enumerate(ctc_targets):
        t = list(t)[:steps]
        ctc[i, :len(t)] = t
        lens[i] = len(t)
    return (np.ascontiguousarray(text_in, np.int32), np.ascontiguousarray(target, np.int32), ctc, lens)
