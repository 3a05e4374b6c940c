"""TEST INFRASTRUCTURE ONLY — CPU oracle of one TRBA INT8-QAT training step.

A numpy restatement of the reference's host training step (later snapshot
src/main.rs:2249-2413, return_main_step) and the model code it drives:

  SE-ResNet QAT backbone  src/qnet.rs:788-1758  (ConvQat, BasicBlock+SE, SEResNetQ)
  BiLSTM stack            src/rnn.rs:101-349    (host fp32 path)
  attention decoder       src/attn.rs:112-500   (teacher-forced forward, backward)
  CTC loss                src/ctc.rs:1-193      (f64 log-space alpha/beta)
  CE loss, clip, steps    src/main.rs:2300-2413, src/opt.rs (Muon + Adam)

Every conv-path operation goes through a CPU implementation of the
reference's backend ABI, called in the reference's order: the reference's own
CPU backend (oracle/_ref/libtrba_ref_omp.so) or our C restatement of it
(oracle/liboracle.so).  Host fp32 parts (SE FCs, BiLSTM, attention, losses,
optimiser) are numpy float32/float64 with the reference's formulas; their
summation order differs from the reference's sequential Rust loops, which is
within the tolerances the parity tests state.

The reference's weight initialisation and smoke data are not seedable
(rand::thread_rng, src/qnet.rs:480-484); this oracle and the GPU build both
take weights from `init_params(seed)` (Glorot-uniform, the reference's
limits) and identical inputs, so "same seed" means "same injected tensors".

Two documented quirks of the reference are kept bit-for-bit in "compat"
mode, because training-loss parity depends on them:
  * the conv weight-gradient GEMM reads its operands in the reference's
    order (transpose_i8 of the NCHW gradient viewed as [rows, Cout], and the
    padded im2col buffer read as [K, rows]) — src/qnet.rs:984-1030;
  * the input gradient of a conv uses the BN-output gradient dy (not the
    BN-backward result) — src/qnet.rs:1068-1080.
"correct" mode (wgrad_mode="correct") computes dW = dX^T col instead.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
F32 = np.float32
BN_EPS = 1e-5
BN_MOMENTUM = F32(0.1)


def a16(x: int) -> int:
    return (x + 15) & ~15


# ---------------------------------------------------------------- backend --
class CpuBackend:
    """A CPU library with the reference backend ABI, called on numpy arrays."""

    def __init__(self, path: str | Path | None = None):
        if path is None:
            ref = HERE / "_ref" / "libtrba_ref_omp.so"
            path = ref if ref.exists() else HERE / "liboracle.so"
        self.path = Path(path)
        self.L = C.CDLL(str(self.path))
        import sys
        sys.path.insert(0, str(REPO / "trba-rust_b200"))
        from ffi import parse_header  # type: ignore
        sys.path.pop(0)
        for name, (res, args) in parse_header((REPO / "include" / "trba_backend.h").read_text()).items():
            if hasattr(self.L, name):
                f = getattr(self.L, name)
                f.restype, f.argtypes = res, args

    def __call__(self, name, *args):
        conv = []
        for a in args:
            if isinstance(a, np.ndarray):
                assert a.flags.c_contiguous
                conv.append(C.c_void_p(a.ctypes.data))
            else:
                conv.append(a)
        getattr(self.L, name)(*conv, None)


# ------------------------------------------------------------- manifest --
@dataclass
class ConvSpec:
    name: str
    cin: int
    cout: int
    kh: int
    kw: int
    sh: int
    sw: int
    ph: int
    pw: int

    @property
    def k(self):
        return self.cin * self.kh * self.kw

    def out_hw(self, h, w):
        return (h + 2 * self.ph - self.kh) // self.sh + 1, (w + 2 * self.pw - self.kw) // self.sw + 1


@dataclass
class Config:
    """Model/data geometry.  Defaults: TRBA-small (fd 128, hidden 64)."""
    fd: int = 128
    hidden: int = 64
    classes: int = 130
    img_h: int = 32
    img_w: int = 160
    max_len: int = 20
    rnn_layers: int = 2
    sos: int = 1
    eos: int = 2
    pad: int = 0
    lr: float = 5.107e-4
    weight_decay: float = 1.9548e-5
    ctc_weight: float = 0.03
    clip_warmup: int = 500
    muon_cap: float = 10.0
    wgrad_mode: str = "compat"
    # Extension (the reference quantises per tensor, src/qnet.rs:316-331):
    # one weight scale per output channel, max |w[row]| / 127.
    wq_per_channel: bool = False

    @property
    def widths(self):
        fd = self.fd
        return [fd // 8, fd // 4, fd // 2, fd // 2, fd, fd]  # src/qnet.rs:1430-1432

    @property
    def steps(self):
        return self.max_len + 1


def block_specs(cfg: Config):
    """(name, in_c, out_c, stride) of every BasicBlock in forward order
    (src/qnet.rs:1435-1455)."""
    w = cfg.widths
    out = [("layer1.0", w[1], w[2], 2), ("layer2.0", w[2], w[3], 1), ("layer2.1", w[3], w[3], 1),
           ("layer3.0", w[3], w[4], 2)]
    out += [(f"layer3.{i}", w[4], w[4], 1) for i in range(1, 5)]
    out += [(f"layer4.{i}", w[5], w[5], 1) for i in range(3)]
    return out


def se_name(block: str) -> str:
    """The reference's checkpoint name of a block's SE layer: layer<i>.<j> ->
    l<i-1>b<j>.se (src/main.rs:985-995)."""
    layer, idx = block.split(".")
    return f"l{int(layer[5:]) - 1}b{idx}.se"


def conv_specs(cfg: Config):
    """Every ConvQat in SEResNetQ::convs_mut order (src/qnet.rs:1457-1471)."""
    w = cfg.widths
    v = [ConvSpec("stem.0", 3, w[0], 3, 3, 1, 1, 1, 1), ConvSpec("stem.3", w[0], w[1], 3, 3, 1, 1, 1, 1)]
    for (name, ic, oc, s) in block_specs(cfg):
        if s != 1 or ic != oc:
            v.append(ConvSpec(f"{name}.downsample.0", ic, oc, 1, 1, s, s, 0, 0))
        v.append(ConvSpec(f"{name}.conv1", ic, oc, 3, 3, s, s, 1, 1))
        v.append(ConvSpec(f"{name}.conv2", oc, oc, 3, 3, 1, 1, 1, 1))
    v.append(ConvSpec("conv_out.0", w[5], w[5], 2, 2, 2, 1, 0, 1))
    v.append(ConvSpec("conv_out.3", w[5], w[5], 2, 2, 1, 1, 0, 0))
    return v


def manifest(cfg: Config):
    """[(name, shape, kind)] in the reference's parameter order (later
    snapshot src/main.rs:954-1030, Model::params_filtered).  kind: 'conv_w'
    (device Muon), 'mat' (host Muon), 'vec' (Adam)."""
    m = []
    for c in conv_specs(cfg):
        m.append((f"{c.name}.w", (c.cout, c.k), "conv_w"))
        m.append((f"{c.name}.gamma", (c.cout,), "vec"))
        m.append((f"{c.name}.beta", (c.cout,), "vec"))
    for (name, ic, oc, s) in block_specs(cfg):
        m.append((f"{se_name(name)}.fc1.w", (oc // 16, oc), "mat"))
        m.append((f"{se_name(name)}.fc2.w", (oc, oc // 16), "mat"))
    H = cfg.hidden
    for li in range(cfg.rnn_layers):
        d = cfg.fd if li == 0 else H
        for dn in ("f", "b"):
            m.append((f"rnn{li}.{dn}.w_ih", (4 * H, d), "mat"))
            m.append((f"rnn{li}.{dn}.b_ih", (4 * H,), "vec"))
            m.append((f"rnn{li}.{dn}.w_hh", (4 * H, H), "mat"))
            m.append((f"rnn{li}.{dn}.b_hh", (4 * H,), "vec"))
        m.append((f"rnn{li}.proj.w", (H, 2 * H), "mat"))
        m.append((f"rnn{li}.proj.b", (H,), "vec"))
    V = cfg.classes
    m += [("attn.i2h.w", (H, H), "mat"), ("attn.h2h.w", (H, H), "mat"), ("attn.h2h.b", (H,), "vec"),
          ("attn.score.w", (1, H), "mat"), ("attn.w_ih", (4 * H, H + V), "mat"), ("attn.b_ih", (4 * H,), "vec"),
          ("attn.w_hh", (4 * H, H), "mat"), ("attn.b_hh", (4 * H,), "vec"), ("attn.gen.w", (V, H), "mat"),
          ("attn.gen.b", (V,), "vec"), ("ctc.w", (V, H), "mat"), ("ctc.b", (V,), "vec")]
    return m


def glorot_limit(name: str, shape, cfg: Config) -> float:
    """The reference's uniform init limits (src/qnet.rs:483, src/rnn.rs:28-29,84,
    src/attn.rs:53-78, src/qnet.rs:109)."""
    H, V = cfg.hidden, cfg.classes
    if name.endswith(".w") and name.count(".") >= 1 and any(name.startswith(c.name) for c in conv_specs(cfg)):
        c = next(c for c in conv_specs(cfg) if name == f"{c.name}.w")
        return math.sqrt(6.0 / (c.k + c.cout * c.kh * c.kw))
    if ".w_ih" in name and name.startswith("rnn"):
        return math.sqrt(6.0 / (shape[1] + 4 * H))
    if ".w_hh" in name and name.startswith("rnn"):
        return math.sqrt(6.0 / (H + 4 * H))
    if name == "attn.w_ih":
        return math.sqrt(6.0 / (H + V + 4 * H))
    if name == "attn.w_hh":
        return math.sqrt(6.0 / (H + 4 * H))
    # LinearF::new(inp, out): sqrt(6/(inp+out)); proj: sqrt(6/(2H+out))
    return math.sqrt(6.0 / (shape[0] + shape[1]))


def init_params(cfg: Config, seed: int) -> dict[str, np.ndarray]:
    """Seeded stand-in for the reference's thread_rng init: Glorot-uniform
    matrices with the reference's limits, BN gamma 1 / beta 0, biases 0."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape, kind in manifest(cfg):
        if kind == "vec":
            out[name] = np.ones(shape, F32) if name.endswith(".gamma") else np.zeros(shape, F32)
        else:
            lim = glorot_limit(name, shape, cfg)
            out[name] = rng.uniform(-lim, lim, size=shape).astype(F32)
    return out


def powi_f32(a: float, n: int) -> np.float32:
    """Rust f32::powi (LLVM's __powisf2): square-and-multiply in f32."""
    r, a = F32(1.0), F32(a)
    while True:
        if n & 1:
            r = F32(r * a)
        n >>= 1
        if n == 0:
            return r
        a = F32(a * a)


def bias_corrections(t: int) -> tuple[float, float]:
    """Adam::bias_correction (src/opt.rs): 1 - beta^t with beta^t in f32."""
    return 1.0 - float(powi_f32(0.9, t)), 1.0 - float(powi_f32(0.999, t))


# ----------------------------------------------------------------- inputs --
def quantise_image(pix: np.ndarray) -> np.ndarray:
    """src/main.rs:881: ((p*2-1)*127).round().clamp(-127,127) with p in [0,1]
    (round half away from zero), s_img = 1/127."""
    v = (pix.astype(F32) * F32(2.0) - F32(1.0)) * F32(127.0)
    r = np.sign(v) * np.floor(np.abs(v) + F32(0.5))
    return np.clip(r, -127, 127).astype(np.int8)


LEN_P50, LEN_P90 = 5, 11


def sample_lengths(rng, b: int, max_len: int) -> np.ndarray:
    """Label lengths with the shape of a handwriting corpus (median 5, p90 11):
    a log-normal fitted to those two quantiles, rounded, clipped to [1, max_len]."""
    mu = math.log(LEN_P50)
    sigma = (math.log(LEN_P90) - mu) / 1.2815515655446004
    l = np.rint(np.exp(rng.normal(mu, sigma, size=b))).astype(np.int64)
    return np.clip(l, 1, max_len)


def make_batch(cfg: Config, b: int, seed: int, fixed_len: int | None = None):
    """Synthetic batch: uniform [0,1] pixels -> int8 image [B,3,H,W]; labels
    of sampled (or fixed) length with tokens U[3, classes); teacher-forcing
    inputs and targets exactly as src/main.rs:2063-2109 builds them."""
    rng = np.random.default_rng(seed)
    pix = rng.random((b, 3, cfg.img_h, cfg.img_w), dtype=np.float32)
    img = quantise_image(pix)
    lens = np.full(b, fixed_len) if fixed_len else sample_lengths(rng, b, cfg.max_len)
    steps = cfg.steps
    text_in = np.full((b, steps), cfg.pad, np.int32)
    target = np.full((b, steps), cfg.pad, np.int32)
    ctc_t = []
    for i in range(b):
        l = int(min(lens[i], cfg.max_len))
        toks = rng.integers(3, cfg.classes, size=l)
        text_in[i, 0] = cfg.sos
        text_in[i, 1:1 + l] = toks
        target[i, :l] = toks
        target[i, l] = cfg.eos
        ctc_t.append(list(toks) + [cfg.eos])
    return img, text_in, target, ctc_t


# ------------------------------------------------------------- host math --
# Host arithmetic.  Every dot product accumulates in f64 and is rounded once
# to f32, and exp / tanh / log are evaluated in f64 and rounded once: the
# results are then the correctly rounded values (ties aside), which the GPU
# build computes the same way, so both produce identical f32 numbers.  The
# reference's sequential f32 loops and f32 libm calls differ from these by a
# few ulps (rayon / OpenMP already make the reference non-reproducible at
# that level).
F64 = np.float64


def dot64(a, b):
    """(a @ b) accumulated in f64, rounded to f32."""
    return (np.asarray(a, F64) @ np.asarray(b, F64)).astype(F32)


def sum64(x, axis=None):
    return np.asarray(x, F64).sum(axis=axis).astype(F32)


def exp32(x):
    return np.exp(np.asarray(x, F32).astype(F64)).astype(F32)


def tanh32(x):
    return np.tanh(np.asarray(x, F32).astype(F64)).astype(F32)


def log32(x):
    return np.log(np.asarray(x, F32).astype(F64)).astype(F32)


def sigmoid(x):
    return (F32(1.0) / (F32(1.0) + exp32(-np.asarray(x, F32)))).astype(F32)


def linear_fwd(x, w, b=None):
    """LinearF::forward (src/qnet.rs:120-138): x w^T (+ b)."""
    y = dot64(x, w.T)
    if b is not None:
        y = (y + b).astype(F32)
    return y


# ------------------------------------------------------------ optimiser --
def adam_vec_step(p, g, m, v, lr, wd, bc1, bc2):
    """Adam for a vector parameter (src/opt.rs:46-65, f64 intermediates, L2
    weight decay folded into the gradient), in place on p, m, v."""
    b1, b2, eps = float(F32(0.9)), float(F32(0.999)), float(F32(1e-8))
    gi = g.astype(np.float64) + float(wd) * p.astype(np.float64)
    m[...] = (b1 * m.astype(np.float64) + (1.0 - b1) * gi).astype(F32)
    v[...] = (b2 * v.astype(np.float64) + (1.0 - b2) * gi * gi).astype(F32)
    mh, vh = m.astype(np.float64) / bc1, v.astype(np.float64) / bc2
    p -= (float(lr) * mh / (np.sqrt(vh) + eps)).astype(F32)


def muon_host_step(p, g, lr, wd, cap):
    """Momentum-free Muon for a matrix parameter (later snapshot src/opt.rs
    muon_step_f32): scale = min(sqrt(min(rows, cols)) / ||g||_F, cap),
    step = lr * sqrt(max(rows, cols)) * scale, decoupled weight decay; in
    place on p (non-finite results become 0)."""
    lr, wd = F32(lr), F32(wd)
    rows, cols = p.shape
    sq = F32((g.astype(F32) * g.astype(F32)).astype(np.float64).sum())
    frob = max(F32(np.sqrt(sq)), F32(1e-8))
    scale = min(F32(np.sqrt(F32(min(rows, cols)))) / frob, F32(cap))
    lr_eff = lr * F32(np.sqrt(F32(max(rows, cols))))
    step = F32(lr_eff * scale)
    dec = F32(F32(1.0) - lr * wd)
    u = (p * dec - step * g).astype(F32)
    p[...] = np.where(np.isfinite(u), u, F32(0))


# ------------------------------------------ per-channel weight quantisation --
def quantize_rows(w, rows_pad, kp):
    """Per-output-channel quantisation (extension of src/qnet.rs:316-331):
    s[r] = max |w[r]| / 127 (1 for an all-zero row, division in f64 rounded
    to f32), q = round-half-away(clamp(f32(w / s[r]), +-127)), padded to the
    GEMM operand [rows_pad, kp]."""
    cout, k = w.shape
    mx = np.abs(w).max(axis=1).astype(np.float64)
    s = np.where(mx > 0, mx / 127.0, 1.0).astype(F32)
    v = (w.astype(np.float64) / s.astype(np.float64)[:, None]).astype(F32)
    v = np.clip(v, F32(-127), F32(127)).astype(np.float64)  # |v| + 0.5 is exact in f64
    q = np.zeros((rows_pad, kp), np.int8)
    q[:cout, :k] = (np.sign(v) * np.floor(np.abs(v) + 0.5)).astype(np.int8)
    return q, s


def grad_input_dequant(dy, wq, w_s, c, b, hi, wi, ho, wo):
    """Input gradient with per-output-channel scales: each input element is
    one f32 running sum over taps (kh, kw outer) and output channels
    (inner) of dy * f32(wq * w_s[oc]), every multiply and add rounded (the
    reference gather's order, cuda/kernels.cu:913-957 of the later snapshot,
    with the dequantised weight in place of the int8 one and no final
    scale)."""
    k = c.cin * c.kh * c.kw
    wdq = (wq[:c.cout, :k].astype(F32) * w_s[:, None]).astype(F32).reshape(c.cout, c.cin, c.kh, c.kw)
    d = dy.reshape(b, c.cout, ho, wo)
    acc = np.zeros((b, c.cin, hi, wi), F32)
    ys, xs = np.arange(hi), np.arange(wi)
    for kh in range(c.kh):
        ny = ys + c.ph - kh
        oky = (ny >= 0) & (ny % c.sh == 0) & (ny // c.sh < ho)
        for kw in range(c.kw):
            nx = xs + c.pw - kw
            okx = (nx >= 0) & (nx % c.sw == 0) & (nx // c.sw < wo)
            if not oky.any() or not okx.any():
                continue
            sh = np.zeros((b, c.cout, hi, wi), F32)  # dy at the tap's output position, 0 where none
            yy, xx = np.nonzero(oky)[0], np.nonzero(okx)[0]
            sh[:, :, yy[:, None], xx[None, :]] = d[:, :, (ny[yy] // c.sh)[:, None], (nx[xx] // c.sw)[None, :]]
            for oc in range(c.cout):
                acc = (acc + (sh[:, oc:oc + 1] * wdq[oc, :, kh, kw][None, :, None, None]).astype(F32)).astype(F32)
    return acc.reshape(-1)


# ---------------------------------------------------------------- oracle --
@dataclass
class ConvState:
    spec: ConvSpec
    wq: np.ndarray = None
    w_s: np.float32 = F32(1.0)


class OracleTrba:
    """The reference training step over a CPU backend.  Parameters live in
    self.p (name -> float32 array); gradients of a step in self.g."""

    def __init__(self, cfg: Config, params: dict[str, np.ndarray], backend: CpuBackend | None = None):
        self.cfg = cfg
        self.be = backend or CpuBackend()
        self.p = {k: v.astype(F32).copy() for k, v in params.items()}
        self.convs = {c.name: ConvState(c) for c in conv_specs(cfg)}
        self.run_mean = {c.name: np.zeros(c.cout, F32) for c in conv_specs(cfg)}
        self.run_var = {c.name: np.ones(c.cout, F32) for c in conv_specs(cfg)}
        self.adam_m = {}
        self.adam_v = {}
        self.t = 0
        for cs in self.convs.values():
            self.requantize(cs)

    # -- weights: device requantize, src/qnet.rs:601-624 -------------------
    def requantize(self, cs: ConvState):
        c = cs.spec
        w = self.p[f"{c.name}.w"]
        mx = np.zeros(1, F32)
        ws = np.zeros(1, F32)
        kp = a16(c.k)
        wq = np.zeros((a16(c.cout), kp), np.int8)
        if self.cfg.wq_per_channel:
            cs.wq, cs.w_s = quantize_rows(w.reshape(c.cout, c.k), a16(c.cout), kp)
            return
        self.be("launch_max_abs_f32", w, mx, w.size)
        self.be("launch_quantize_pad_i8", w, mx, ws, wq, c.cout, c.k, kp)
        cs.wq, cs.w_s = wq, F32(ws[0])

    # -- quant helpers: src/qnet.rs:1089-1112 ------------------------------
    def _scale(self, v):
        mx = np.zeros(1, F32)
        self.be("launch_reduce_max_abs", v, v.size, mx)
        return max(F32(mx[0] / F32(127.0)), F32(1e-12))

    def relu_quant(self, y):
        s = self._scale(y)
        q = np.zeros(y.size, np.int8)
        self.be("launch_relu_quant", y, y.size, float(s), q)
        return q, s

    def quant(self, v):
        s = self._scale(v)
        q = np.zeros(v.size, np.int8)
        self.be("launch_quant_f32_i8", v, v.size, float(s), q)
        return q, s

    def dequant(self, q, s):
        x = np.zeros(q.size, F32)
        self.be("launch_dequant_i8_f32", q, q.size, float(s), x)
        return x

    def mask(self, q, d):
        qv = self.dequant(q, 1.0)
        out = np.zeros(d.size, F32)
        self.be("launch_mask_relu_bwd", qv, d, d.size, out)
        return out

    # -- ConvQat::forward, src/qnet.rs:788-916 -----------------------------
    def conv_fwd(self, name, q_in, s_in, b, h, w, train=True):
        cs = self.convs[name]
        c = cs.spec
        ho, wo = c.out_hw(h, w)
        rows, k = b * ho * wo, c.k
        kp, rp = a16(k), a16(rows)
        col = np.zeros(rp * kp, np.int8)
        self.be("launch_im2col_pad", q_in, col, b, c.cin, h, w, c.kh, c.kw, c.sh, c.sw, c.ph, c.pw, ho, wo, kp)
        acc = np.zeros(rows * c.cout, np.int32)
        self.be("launch_gemm_int8", col, cs.wq, acc, rows, c.cout, k)
        n = b * c.cout * ho * wo
        x = np.zeros(n, F32)
        if self.cfg.wq_per_channel:  # x = acc * (s_in * w_s[n]), NCHW
            sc = (F32(s_in) * cs.w_s).astype(F32)
            x[...] = (acc.reshape(b, ho * wo, c.cout).astype(F32) * sc).astype(F32).transpose(0, 2, 1).reshape(-1)
        else:
            self.be("launch_epilogue_f32", acc, c.cout, float(F32(s_in) * cs.w_s), x, c.cout, ho, wo, n)
        mean, var = np.zeros(c.cout, F32), np.zeros(c.cout, F32)
        if train:
            self.be("launch_bn_stats", x, b, c.cout, ho * wo, mean, var)
        else:  # inference: running statistics (src/qnet.rs:871-876)
            mean[:], var[:] = self.run_mean[name], self.run_var[name]
        y = np.zeros(n, F32)
        self.be("launch_bn_apply", x, mean, var, self.p[f"{name}.gamma"], self.p[f"{name}.beta"], BN_EPS, y,
                c.cout, ho * wo, n)
        return dict(name=name, b=b, h=h, w=w, ho=ho, wo=wo, s_in=F32(s_in), q_in=q_in, x=x, y=y, mean=mean,
                    var=var, col=col)

    # -- ConvQat::backward, src/qnet.rs:918-1083 ---------------------------
    def conv_bwd(self, dy, tr, need_dx=True):
        name = tr["name"]
        cs = self.convs[name]
        c = cs.spec
        b, ho, wo, hi, wi = tr["b"], tr["ho"], tr["wo"], tr["h"], tr["w"]
        rows, hw, k = b * ho * wo, ho * wo, c.k
        kp, rp = a16(k), a16(rows)
        n_out = b * c.cout * hw
        sdy, sdxh = np.zeros(c.cout, F32), np.zeros(c.cout, F32)
        self.be("launch_bn_bwd_sums", dy, tr["x"], tr["mean"], tr["var"], BN_EPS, c.cout, hw, n_out, sdy, sdxh)
        dx = np.zeros(n_out, F32)
        self.be("launch_bn_bwd_dx", dy, tr["x"], tr["mean"], tr["var"], self.p[f"{name}.gamma"], sdy, sdxh, BN_EPS,
                c.cout, hw, n_out, b * hw, dx)
        self.g[f"{name}.beta"] += sdy
        self.g[f"{name}.gamma"] += sdxh
        qdx, s_dx = self.quant(dx)
        gw = np.zeros(c.cout * k, np.int32)
        if self.cfg.wgrad_mode == "compat":
            # transpose_i8 writes [Cout, rows] with ld rows; the GEMM reads ld
            # align16(rows) (identical when rows % 16 == 0, true at every
            # benchmark size; unwritten tail bytes are zero here).
            qdx_t = np.zeros(a16(c.cout) * rp, np.int8)
            self.be("launch_transpose_i8", qdx, rows, c.cout, qdx_t)
            self.be("launch_gemm_int8", qdx_t, tr["col"], gw, c.cout, k, rows)
        else:
            # dW[o, n] = sum_r dX[r, o] col[r, n], dX from the NCHW gradient
            A = np.zeros((a16(c.cout), rp), np.int8)
            A[:c.cout, :rows] = qdx.reshape(b, c.cout, hw).transpose(1, 0, 2).reshape(c.cout, rows)
            Bt = np.zeros((a16(k), rp), np.int8)
            Bt[:k, :rows] = tr["col"].reshape(rp, kp)[:rows, :k].T
            self.be("launch_gemm_int8", np.ascontiguousarray(A), np.ascontiguousarray(Bt), gw, c.cout, k, rows)
        deq = F32(s_dx) * tr["s_in"]
        g = self.g[f"{name}.w"].reshape(-1)
        self.be("launch_grad_accum_i32", gw, g, float(deq), g.size)
        if not need_dx:
            return None
        gi = np.zeros(b * c.cin * hi * wi, F32)
        if self.cfg.wq_per_channel:
            return grad_input_dequant(dy, cs.wq, cs.w_s, c, b, hi, wi, ho, wo)
        self.be("launch_conv_backward_grad_input_i8", dy, cs.wq, kp, float(cs.w_s), gi, b, c.cin, hi, wi, c.cout,
                c.kh, c.kw, c.sh, c.sw, c.ph, c.pw, ho, wo)
        return gi

    # -- BasicBlock::forward, src/qnet.rs:1182-1271 ------------------------
    def block_fwd(self, bname, has_ds, q_in, s_in, b, h, w, train=True):
        cout = self.convs[f"{bname}.conv2"].spec.cout
        ds = self.conv_fwd(f"{bname}.downsample.0", q_in, s_in, b, h, w, train) if has_ds else None
        f1 = self.conv_fwd(f"{bname}.conv1", q_in, s_in, b, h, w, train)
        q1, s1 = self.relu_quant(f1["y"])
        f2 = self.conv_fwd(f"{bname}.conv2", q1, s1, b, f1["ho"], f1["wo"], train)
        hw = f2["ho"] * f2["wo"]
        n_out = b * cout * hw
        pooled = np.zeros(b * cout, F32)
        self.be("launch_avgpool_hw", f2["y"], cout, hw, b, pooled)
        pre1 = linear_fwd(pooled.reshape(b, cout), self.p[f"{se_name(bname)}.fc1.w"])
        h1 = np.maximum(pre1, F32(0)).astype(F32)
        pre2 = linear_fwd(h1, self.p[f"{se_name(bname)}.fc2.w"])
        gate = sigmoid(pre2).reshape(-1)
        yse = np.zeros(n_out, F32)
        self.be("launch_mul_gate", f2["y"], gate, cout, hw, n_out, yse)
        z = np.zeros(n_out, F32)
        if ds is not None:
            self.be("launch_add_f32", yse, ds["y"], n_out, z)
        else:
            idv = self.dequant(q_in, s_in)
            self.be("launch_add_f32", yse, idv, n_out, z)
        q_out, s_z = self.relu_quant(z)
        tr = dict(name=bname, c1=f1, c2=f2, ds=ds, q1=q1, s1=s1, y2=f2["y"], gate=gate, pooled=pooled, h1=h1, b=b,
                  c=cout, ho=f2["ho"], wo=f2["wo"])
        return q_out, s_z, tr

    # -- BasicBlock::backward, src/qnet.rs:1275-1355 -----------------------
    def block_bwd(self, dq_out, s_dq, q_out, tr):
        b, c, hw = tr["b"], tr["c"], tr["ho"] * tr["wo"]
        n_out = b * c * hw
        bname = tr["name"]
        gvz = self.dequant(dq_out, s_dq)
        dz = self.mask(q_out, gvz)
        dy2 = np.zeros(n_out, F32)
        self.be("launch_mul_gate", dz, tr["gate"], c, hw, n_out, dy2)
        prod = np.zeros(n_out, F32)
        self.be("launch_mul_f32", dz, tr["y2"], n_out, prod)
        pm = np.zeros(b * c, F32)
        self.be("launch_avgpool_hw", prod, c, hw, b, pm)
        dgate = (pm * F32(hw)).astype(F32)
        gate = tr["gate"]
        dpre2 = (dgate * gate * (F32(1.0) - gate)).astype(F32).reshape(b, c)
        w2, w1 = self.p[f"{se_name(bname)}.fc2.w"], self.p[f"{se_name(bname)}.fc1.w"]
        self.g[f"{se_name(bname)}.fc2.w"] += dot64(dpre2.T, tr["h1"])
        dh1 = dot64(dpre2, w2)
        dpre1 = np.where(tr["h1"] > 0, dh1, F32(0)).astype(F32)
        self.g[f"{se_name(bname)}.fc1.w"] += dot64(dpre1.T, tr["pooled"].reshape(b, c))
        dpooled = dot64(dpre1, w1).reshape(-1)
        apb = np.zeros(n_out, F32)
        self.be("launch_avgpool_hw_backward", dpooled, c, hw, b, apb)
        dy2f = np.zeros(n_out, F32)
        self.be("launch_add_f32", dy2, apb, n_out, dy2f)
        gv1 = self.conv_bwd(dy2f, tr["c2"])
        dy1 = self.mask(tr["q1"], gv1)
        gi = self.conv_bwd(dy1, tr["c1"])
        total = np.zeros(gi.size, F32)
        if tr["ds"] is not None:
            dxds = self.conv_bwd(dz, tr["ds"])
            self.be("launch_add_f32", gi, dxds, gi.size, total)
        else:
            self.be("launch_add_f32", gi, dz, gi.size, total)
        return total

    # -- SEResNetQ::forward / backward, src/qnet.rs:1533-1737 ---------------
    def cnn_fwd(self, img, b, train=True):
        cfg = self.cfg
        h, w = cfg.img_h, cfg.img_w
        s_img = F32(1.0) / F32(127.0)
        chain = []
        f0 = self.conv_fwd("stem.0", img, s_img, b, h, w, train)
        q0, s0 = self.relu_quant(f0["y"])
        f1 = self.conv_fwd("stem.3", q0, s0, b, h, w, train)
        q1, s1 = self.relu_quant(f1["y"])
        c1 = self.convs["stem.3"].spec.cout
        qp = np.zeros(b * c1 * (h // 2) * (w // 2), np.int8)
        self.be("launch_maxpool2x2_forward_i8", q1, qp, b, c1, h, w)
        h, w = h // 2, w // 2
        q, s = qp, s1
        blocks = []
        for (name, ic, oc, st) in block_specs(cfg):
            q, s, tr = self.block_fwd(name, st != 1 or ic != oc, q, s, b, h, w, train)
            h, w = tr["ho"], tr["wo"]
            blocks.append(tr)
            chain.append((q, s))
        fo0 = self.conv_fwd("conv_out.0", q, s, b, h, w, train)
        qo0, so0 = self.relu_quant(fo0["y"])
        fo1 = self.conv_fwd("conv_out.3", qo0, so0, b, fo0["ho"], fo0["wo"], train)
        qo1, so1 = self.relu_quant(fo1["y"])
        hf, wf = fo1["ho"], fo1["wo"]
        fv = self.dequant(qo1, so1)
        feat = np.zeros(b * wf * cfg.fd, F32)
        self.be("launch_meanpool_h", fv, cfg.fd, hf, wf, b, feat)
        trace = dict(f0=f0, f1=f1, q0=q0, s0=s0, q1=q1, s1=s1, blocks=blocks, chain=chain, fo0=fo0, fo1=fo1,
                     qo0=qo0, so0=so0, qo1=qo1, so1=so1, hf=hf, wf=wf, b=b, hpool=cfg.img_h, wpool=cfg.img_w)
        return feat, trace

    def cnn_bwd(self, d_feat, tr):
        cfg, b = self.cfg, tr["b"]
        hf, wf = tr["hf"], tr["wf"]
        no1 = b * cfg.fd * hf * wf
        dv = np.zeros(no1, F32)
        self.be("launch_meanpool_h_backward", d_feat, cfg.fd, hf, wf, b, dv)
        self.be("cuda_scale_vector", dv, float(tr["so1"]), no1)
        dy1 = self.mask(tr["qo1"], dv)
        gv = self.conv_bwd(dy1, tr["fo1"])
        dy0 = self.mask(tr["qo0"], gv)
        gv = self.conv_bwd(dy0, tr["fo0"])
        for bi in range(len(tr["blocks"]) - 1, -1, -1):
            q_out, s_out = tr["chain"][bi]
            self.be("cuda_scale_vector", gv, float(s_out), gv.size)
            dqi, s_dq = self.quant(gv)
            gv = self.block_bwd(dqi, s_dq, q_out, tr["blocks"][bi])
        self.be("cuda_scale_vector", gv, float(tr["s1"]), gv.size)
        c1 = self.convs["stem.3"].spec.cout
        n1 = b * c1 * tr["hpool"] * tr["wpool"]
        dpre = np.zeros(n1, F32)
        self.be("launch_maxpool2x2_backward_i8", tr["q1"], gv, dpre, b, c1, tr["hpool"], tr["wpool"])
        dyc1 = self.mask(tr["q1"], dpre)
        gvc0 = self.conv_bwd(dyc1, tr["f1"])
        dyc0 = self.mask(tr["q0"], gvc0)
        # stem.0's input gradient (the image gradient) is discarded by the
        # reference (src/qnet.rs:1736): only its weight/BN gradients matter.
        self.conv_bwd(dyc0, tr["f0"], need_dx=False)

    def update_running_stats(self, tr):
        """src/qnet.rs:1740-1757 with BatchNorm::update_running (:63-68)."""
        fs = [tr["f0"], tr["f1"]]
        for bt in tr["blocks"]:
            if bt["ds"] is not None:
                fs.append(bt["ds"])
            fs += [bt["c1"], bt["c2"]]
        fs += [tr["fo0"], tr["fo1"]]
        for f in fs:
            n = f["name"]
            self.run_mean[n] = ((F32(1) - BN_MOMENTUM) * self.run_mean[n] + BN_MOMENTUM * f["mean"]).astype(F32)
            self.run_var[n] = ((F32(1) - BN_MOMENTUM) * self.run_var[n] + BN_MOMENTUM * f["var"]).astype(F32)

    # -- BiLSTM, src/rnn.rs:101-349 ----------------------------------------
    def lstm_dir(self, pre, x, b, t, rev):
        w_ih, b_ih, w_hh, b_hh = (self.p[pre + s] for s in (".w_ih", ".b_ih", ".w_hh", ".b_hh"))
        H = w_hh.shape[1]
        xg = dot64(x.reshape(b * t, -1), w_ih.T).reshape(b, t, 4 * H)  # [B, T, 4H]
        gates = np.zeros((t, b, 4 * H), F32)
        cs = np.zeros((t, b, H), F32)
        hs = np.zeros((t, b, H), F32)
        hprev = np.zeros((t, b, H), F32)
        c_prev = np.zeros((b, H), F32)
        h_prev = np.zeros((b, H), F32)
        bsum = (b_ih + b_hh).astype(F32)
        for step in range(t):
            tt = t - 1 - step if rev else step
            g = ((bsum + xg[:, tt, :]) + dot64(h_prev, w_hh.T)).astype(F32)
            ig, fg = sigmoid(g[:, :H]), sigmoid(g[:, H:2 * H])
            cg, og = tanh32(g[:, 2 * H:3 * H]), sigmoid(g[:, 3 * H:])
            c = (fg * c_prev + ig * cg).astype(F32)
            hh = (og * tanh32(c)).astype(F32)
            gates[step] = np.concatenate([ig, fg, cg, og], axis=1)
            cs[step], hs[step], hprev[step] = c, hh, h_prev
            c_prev, h_prev = c, hh
        return dict(gates=gates, c=cs, h=hs, hprev=hprev)

    def bilstm_layer_fwd(self, li, x, b, t):
        f = self.lstm_dir(f"rnn{li}.f", x, b, t, False)
        r = self.lstm_dir(f"rnn{li}.b", x, b, t, True)
        H = self.cfg.hidden
        cat = np.zeros((b, t, 2 * H), F32)
        cat[:, :, :H] = f["h"].transpose(1, 0, 2)
        cat[:, :, H:] = r["h"][::-1].transpose(1, 0, 2)
        y = linear_fwd(cat.reshape(b * t, 2 * H), self.p[f"rnn{li}.proj.w"], self.p[f"rnn{li}.proj.b"])
        return y.reshape(-1), dict(x=x, f=f, r=r, cat=cat, b=b, t=t)

    def lstm_dir_bwd(self, pre, dh_out, tr, trc, rev, true_cell_grad=False):
        """Backward through one direction.  The reference carries the cell
        gradient into the previous step as dc and multiplies it there by that
        step's own forget gate (src/rnn.rs:267, later snapshot); the chain
        rule multiplies by the forget gate of the step the gradient comes
        from.  true_cell_grad=True computes the latter (for the
        finite-difference checks); the default keeps the reference's."""
        b, t = tr["b"], tr["t"]
        w_ih, w_hh = self.p[pre + ".w_ih"], self.p[pre + ".w_hh"]
        H, D = w_hh.shape[1], w_ih.shape[1]
        x = tr["x"].reshape(b, t, D)
        dg_all = np.zeros((b, t, 4 * H), F32)    # by time position
        hp_all = np.zeros((b, t, H), F32)
        dc_next = np.zeros((b, H), F32)
        dh_next = np.zeros((b, H), F32)
        for step in range(t - 1, -1, -1):
            tt = t - 1 - step if rev else step
            gr, c = trc["gates"][step], trc["c"][step]
            c_prev = trc["c"][step - 1] if step else np.zeros((b, H), F32)
            ig, fg, cg, og = gr[:, :H], gr[:, H:2 * H], gr[:, 2 * H:3 * H], gr[:, 3 * H:]
            tc = tanh32(c)
            dh = (dh_out[step] + dh_next).astype(F32)
            if true_cell_grad:
                dc = (dh * og * (F32(1) - tc * tc) + dc_next).astype(F32)
            else:
                dc = (dh * og * (F32(1) - tc * tc) + dc_next * fg).astype(F32)
            dg = np.concatenate([dc * cg * ig * (F32(1) - ig), dc * c_prev * fg * (F32(1) - fg),
                                 dc * ig * (F32(1) - cg * cg), dh * tc * og * (F32(1) - og)], axis=1).astype(F32)
            dc_next = (dc * fg).astype(F32) if true_cell_grad else dc
            dg_all[:, tt] = dg
            hp_all[:, tt] = trc["hprev"][step]
            dh_next = dot64(dg, w_hh)
        dg2 = dg_all.reshape(b * t, 4 * H)
        gb = sum64(dg2, axis=0)
        self.g[pre + ".w_ih"] += dot64(dg2.T, x.reshape(b * t, D))
        self.g[pre + ".w_hh"] += dot64(dg2.T, hp_all.reshape(b * t, H))
        self.g[pre + ".b_ih"] += gb
        self.g[pre + ".b_hh"] += gb
        return dot64(dg2, w_ih).reshape(-1)

    def bilstm_layer_bwd(self, li, dy, tr):
        b, t, H = tr["b"], tr["t"], self.cfg.hidden
        dy = dy.reshape(b * t, H)
        pw = self.p[f"rnn{li}.proj.w"]
        dcat = dot64(dy, pw).reshape(b, t, 2 * H)
        self.g[f"rnn{li}.proj.w"] += dot64(dy.T, tr["cat"].reshape(b * t, 2 * H))
        self.g[f"rnn{li}.proj.b"] += sum64(dy, axis=0)
        dh_f = dcat[:, :, :H].transpose(1, 0, 2)
        dh_b = dcat[:, ::-1, H:].transpose(1, 0, 2)
        dx1 = self.lstm_dir_bwd(f"rnn{li}.f", np.ascontiguousarray(dh_f), tr, tr["f"], False)
        dx2 = self.lstm_dir_bwd(f"rnn{li}.b", np.ascontiguousarray(dh_b), tr, tr["r"], True)
        return (dx1 + dx2).astype(F32)

    # -- attention decoder, src/attn.rs:119-500 -----------------------------
    def attn_fwd(self, enc, text_in, b, t):
        cfg = self.cfg
        H, V, steps = cfg.hidden, cfg.classes, text_in.shape[1]
        P = self.p
        bh = enc.reshape(b, t, H)
        proj_h = dot64(bh.reshape(b * t, H), P["attn.i2h.w"].T).reshape(b, t, H)
        h = np.zeros((b, H), F32)
        cc = np.zeros((b, H), F32)
        tr = dict(tanh=np.zeros((steps, b, t, H), F32), alpha=np.zeros((steps, b, t), F32),
                  cell_in=np.zeros((steps, b, H + V), F32), gates=np.zeros((steps, b, 4 * H), F32),
                  hs=np.zeros((steps, b, H), F32), cs=np.zeros((steps, b, H), F32))
        scw = P["attn.score.w"].reshape(H)
        wc, wtok = P["attn.w_ih"][:, :H], P["attn.w_ih"][:, H:]
        bsum = (P["attn.b_ih"] + P["attn.b_hh"]).astype(F32)
        for st in range(steps):
            phh = linear_fwd(h, P["attn.h2h.w"], P["attn.h2h.b"])
            tn = tanh32(proj_h + phh[:, None, :])
            e = dot64(tn, scw)
            ex = exp32(e - e.max(axis=1, keepdims=True))
            alpha = (ex / sum64(ex, axis=1)[:, None]).astype(F32)
            ctx = np.einsum("bt,btk->bk", alpha.astype(F64), bh.astype(F64)).astype(F32)
            tok = text_in[:, st]
            ci = np.zeros((b, H + V), F32)
            ci[:, :H] = ctx
            ci[np.arange(b), H + tok] = F32(1.0)
            pre = (((bsum + dot64(ctx, wc.T)) + wtok[:, tok].T) + dot64(h, P["attn.w_hh"].T)).astype(F32)
            ig, fg = sigmoid(pre[:, :H]), sigmoid(pre[:, H:2 * H])
            cg, og = tanh32(pre[:, 2 * H:3 * H]), sigmoid(pre[:, 3 * H:])
            cc = (fg * cc + ig * cg).astype(F32)
            h = (og * tanh32(cc)).astype(F32)
            tr["tanh"][st], tr["alpha"][st], tr["cell_in"][st] = tn, alpha, ci
            tr["gates"][st] = np.concatenate([ig, fg, cg, og], axis=1)
            tr["hs"][st], tr["cs"][st] = h, cc
        logits_sb = linear_fwd(tr["hs"].reshape(steps * b, H), P["attn.gen.w"], P["attn.gen.b"])
        logits = logits_sb.reshape(steps, b, V).transpose(1, 0, 2).copy()  # [B, steps, V]
        tr.update(bh=bh, proj_h=proj_h, b=b, t=t, steps=steps)
        return logits, tr

    # -- AttentionDecoder::greedy_decode, src/attn.rs:368-447 --------------
    def greedy_decode(self, enc, b, t):
        """Greedy decoding from sos: the argmax token (first maximum) is fed
        back; decoding stops after the first step at which every sample of the
        batch produced eos; eos tokens are not emitted, tokens after a
        sample's eos are (as in the reference).  Returns (per-sample token
        lists, per-step argmax tokens [steps, b])."""
        cfg = self.cfg
        H, V, steps = cfg.hidden, cfg.classes, cfg.steps
        P = self.p
        bh = enc.reshape(b, t, H)
        proj_h = dot64(bh.reshape(b * t, H), P["attn.i2h.w"].T).reshape(b, t, H)
        h = np.zeros((b, H), F32)
        cc = np.zeros((b, H), F32)
        scw = P["attn.score.w"].reshape(H)
        wc, wtok = P["attn.w_ih"][:, :H], P["attn.w_ih"][:, H:]
        bsum = (P["attn.b_ih"] + P["attn.b_hh"]).astype(F32)
        tok = np.full(b, cfg.sos, np.int64)
        out = [[] for _ in range(b)]
        step_tok = np.full((steps, b), -1, np.int32)
        for st in range(steps):
            phh = linear_fwd(h, P["attn.h2h.w"], P["attn.h2h.b"])
            tn = tanh32(proj_h + phh[:, None, :])
            e = dot64(tn, scw)
            ex = exp32(e - e.max(axis=1, keepdims=True))
            alpha = (ex / sum64(ex, axis=1)[:, None]).astype(F32)
            ctx = np.einsum("bt,btk->bk", alpha.astype(F64), bh.astype(F64)).astype(F32)
            pre = (((bsum + dot64(ctx, wc.T)) + wtok[:, tok].T) + dot64(h, P["attn.w_hh"].T)).astype(F32)
            ig, fg = sigmoid(pre[:, :H]), sigmoid(pre[:, H:2 * H])
            cg, og = tanh32(pre[:, 2 * H:3 * H]), sigmoid(pre[:, 3 * H:])
            cc = (fg * cc + ig * cg).astype(F32)
            h = (og * tanh32(cc)).astype(F32)
            logits = linear_fwd(h, P["attn.gen.w"], P["attn.gen.b"])
            best = np.argmax(logits, axis=1)
            step_tok[st] = best
            all_eos = True
            for bi in range(b):
                if best[bi] == cfg.eos:
                    continue
                all_eos = False
                out[bi].append(int(best[bi]))
            tok = best
            if all_eos:
                break
        return out, step_tok

    def infer(self, img):
        """run_inference (later snapshot src/main.rs:2690): the CNN with BN
        running statistics, the BiLSTM stack, greedy attention decoding."""
        b = img.shape[0]
        feat, ctr = self.cnn_fwd(np.ascontiguousarray(img.reshape(-1)), b, train=False)
        t = ctr["wf"]
        x = feat
        for li in range(self.cfg.rnn_layers):
            x, _ = self.bilstm_layer_fwd(li, x, b, t)
        return self.greedy_decode(x.reshape(b, t, self.cfg.hidden), b, t)

    def attn_bwd(self, d_logits, tr, true_cell_grad=False):
        """Backward through the decoder; true_cell_grad as in lstm_dir_bwd
        (the reference's decoder cell, src/attn.rs:314 of the later snapshot,
        carries the cell gradient the same way as its BiLSTM)."""
        cfg, P, G = self.cfg, self.p, self.g
        b, t, steps = tr["b"], tr["t"], tr["steps"]
        H, V = cfg.hidden, cfg.classes
        dyg = d_logits.reshape(b, steps, V).transpose(1, 0, 2).reshape(steps * b, V)
        hs = tr["hs"].reshape(steps * b, H)
        G["attn.gen.w"] += dot64(dyg.T, hs)
        G["attn.gen.b"] += sum64(dyg, axis=0)
        d_out_hid = dot64(dyg, P["attn.gen.w"]).reshape(steps, b, H)
        dh_next = np.zeros((b, H), F32)
        dc_next = np.zeros((b, H), F32)
        d_proj_h = np.zeros((b, t, H), F32)
        d_bh = np.zeros((b, t, H), F32)
        scw = P["attn.score.w"].reshape(H)
        wc = P["attn.w_ih"][:, :H]
        zeros = np.zeros((b, H), F32)
        dg_all = np.zeros((steps, b, 4 * H), F32)
        de_all = np.zeros((steps, b, t), F32)
        dphh_all = np.zeros((steps, b, H), F32)
        for st in range(steps - 1, -1, -1):
            g = tr["gates"][st]
            c_prev = tr["cs"][st - 1] if st else zeros
            ig, fg, cg, og = g[:, :H], g[:, H:2 * H], g[:, 2 * H:3 * H], g[:, 3 * H:]
            tc = tanh32(tr["cs"][st])
            dh = (d_out_hid[st] + dh_next).astype(F32)
            if true_cell_grad:
                dc = (dh * og * (F32(1) - tc * tc) + dc_next).astype(F32)
            else:
                dc = (dh * og * (F32(1) - tc * tc) + dc_next * fg).astype(F32)
            dg = np.concatenate([dc * cg * ig * (F32(1) - ig), dc * c_prev * fg * (F32(1) - fg),
                                 dc * ig * (F32(1) - cg * cg), dh * tc * og * (F32(1) - og)], axis=1).astype(F32)
            dc_next = (dc * fg).astype(F32) if true_cell_grad else dc
            dg_all[st] = dg
            dctx = dot64(dg, wc)
            dh_prev = dot64(dg, P["attn.w_hh"])
            alpha = tr["alpha"][st]
            da = np.einsum("bk,btk->bt", dctx.astype(F64), tr["bh"].astype(F64)).astype(F32)
            d_bh += (alpha[:, :, None] * dctx[:, None, :]).astype(F32)
            dot = np.einsum("bt,bt->b", alpha.astype(F64), da.astype(F64)).astype(F32)
            de = (alpha * (da - dot[:, None])).astype(F32)  # [B, T]
            de_all[st] = de
            tn = tr["tanh"][st]
            dtn = (de[:, :, None] * scw[None, None, :] * (F32(1) - tn * tn)).astype(F32)
            d_proj_h += dtn
            dprojhh = sum64(dtn, axis=1)
            dphh_all[st] = dprojhh
            dh_next = (dh_prev + dot64(dprojhh, P["attn.h2h.w"])).astype(F32)
        R = steps * b
        dg2 = dg_all.reshape(R, 4 * H)
        sdg = sum64(dg2, axis=0)
        G["attn.b_ih"] += sdg
        G["attn.b_hh"] += sdg
        G["attn.w_ih"] += dot64(dg2.T, tr["cell_in"].reshape(R, H + V))
        hs_prev = tr["hs"].reshape(R, H)[:R - b]  # h_prev of steps 1.. (zero at step 0)
        G["attn.w_hh"] += dot64(dg2[b:].T, hs_prev)
        dp2 = dphh_all.reshape(R, H)
        G["attn.h2h.w"] += dot64(dp2[b:].T, hs_prev)
        G["attn.h2h.b"] += sum64(dp2, axis=0)
        G["attn.score.w"] += dot64(de_all.reshape(1, R * t), tr["tanh"].reshape(R * t, H))
        dph = d_proj_h.reshape(b * t, H)
        G["attn.i2h.w"] += dot64(dph.T, tr["bh"].reshape(b * t, H))
        d_bh = (dot64(dph, P["attn.i2h.w"]) + d_bh.reshape(b * t, H)).astype(F32)
        return d_bh.reshape(-1)

    # -- CTC, src/ctc.rs:1-193 ----------------------------------------------
    @staticmethod
    def ctc_loss_backward(logits, b, t, V, targets, blank=0):
        lg = logits.reshape(b * t, V)
        mx = lg.max(axis=1, keepdims=True)
        e = np.exp((lg - mx).astype(np.float64))
        se = e.sum(axis=1, keepdims=True)
        lp32 = (lg.astype(np.float64) - mx.astype(np.float64) - np.log(se)).astype(F32)
        lp = lp32.astype(np.float64)
        grad = np.zeros((b * t, V), F32)
        counted = max(1, sum(1 for tg in targets if len(tg) and t >= len(tg) + 1))
        n = float(counted)
        total = 0.0
        NEG = -np.inf

        def logadd(a, c):
            if a == NEG:
                return c
            if c == NEG:
                return a
            return a + math.log1p(math.exp(c - a)) if a > c else c + math.log1p(math.exp(a - c))

        for bi in range(b):
            tg = targets[bi]
            L = len(tg)
            if L == 0 or t < L + 1:
                continue
            ext = [blank]
            for x in tg:
                ext += [x, blank]
            S = len(ext)
            lpb = lp[bi * t:(bi + 1) * t]
            al = np.full((t, S), NEG)
            al[0, 0] = lpb[0, ext[0]]
            if S > 1:
                al[0, 1] = lpb[0, ext[1]]
            for tt in range(1, t):
                for si in range(S):
                    best = al[tt - 1, si]
                    if si > 0:
                        best = logadd(best, al[tt - 1, si - 1])
                    if si >= 2 and ext[si - 2] != ext[si]:
                        best = logadd(best, al[tt - 1, si - 2])
                    al[tt, si] = best + lpb[tt, ext[si]]
            loss = -logadd(al[t - 1, S - 1], al[t - 1, S - 2])
            if not math.isfinite(loss):
                continue
            be = np.full((t, S), NEG)
            be[t - 1, S - 1] = 0.0
            if S > 1:
                be[t - 1, S - 2] = 0.0
            for tt in range(t - 2, -1, -1):
                row = lpb[tt + 1]
                for si in range(S):
                    best = be[tt + 1, si] + row[ext[si]]
                    if si + 1 < S:
                        best = logadd(best, be[tt + 1, si + 1] + row[ext[si + 1]])
                    if si + 2 < S and ext[si + 2] != ext[si]:
                        best = logadd(best, be[tt + 1, si + 2] + row[ext[si + 2]])
                    be[tt, si] = best
            total += loss / L
            gamma = np.zeros((t, V))
            for tt in range(t):
                for si in range(S):
                    gamma[tt, ext[si]] += math.exp(al[tt, si] + be[tt, si] + loss)
            scale = 1.0 / (L * n)
            p = exp32(lp32[bi * t:(bi + 1) * t]).astype(np.float64)
            grad[bi * t:(bi + 1) * t] = ((p - gamma) * scale).astype(F32)
        return total / n, grad.reshape(-1)

    # -- the step: src/main.rs:2249-2413 ------------------------------------
    def train_step(self, img, text_in, target, ctc_targets, optimize: bool = True):
        """One step (src/main.rs:2249-2413): forward, losses, backward into
        self.g and, unless optimize is False (data-parallel callers average
        self.g across ranks first), the optimiser step."""
        cfg = self.cfg
        b = img.shape[0]
        H, V, steps = cfg.hidden, cfg.classes, cfg.steps
        cw = F32(cfg.ctc_weight)
        self.g = {k: np.zeros_like(v) for k, v in self.p.items()}
        feat, ctr = self.cnn_fwd(np.ascontiguousarray(img.reshape(-1)), b)
        self.update_running_stats(ctr)
        t = ctr["wf"]
        x = feat
        rtr = []
        for li in range(cfg.rnn_layers):
            x, tr = self.bilstm_layer_fwd(li, x, b, t)
            rtr.append(tr)
        enc = x.reshape(b, t, H)
        logits, atr = self.attn_fwd(enc, text_in, b, t)
        ctc_logits = linear_fwd(enc.reshape(b * t, H), self.p["ctc.w"], self.p["ctc.b"])
        # attention CE with ignore PAD (src/main.rs:2300-2328)
        lg = logits.reshape(b * steps, V)
        tgt = target.reshape(-1)
        keep = tgt != cfg.pad
        count = int(keep.sum())
        mx = lg.max(axis=1, keepdims=True)
        ex = exp32(lg - mx)
        s = sum64(ex, axis=1)[:, None]
        pr = (ex / s).astype(F32)
        attn_loss = float(-log32(pr[keep, tgt[keep]]).astype(np.float64).sum())
        d_logits = pr.copy()
        d_logits[np.arange(b * steps), tgt] -= F32(1.0)
        d_logits[~keep] = 0
        count = max(count, 1)
        attn_loss /= count
        d_logits = (d_logits * F32((F32(1.0) - cw) / F32(count))).astype(F32)
        ctc_loss, d_ctc = self.ctc_loss_backward(ctc_logits, b, t, V, ctc_targets, 0)
        d_ctc = (d_ctc * cw).astype(F32)
        total = float(float(F32(1.0) - cw) * attn_loss + float(cw) * ctc_loss)
        self.debug = dict(feat=feat, enc=enc.reshape(-1), logits=logits.transpose(1, 0, 2).reshape(-1),
                          dlogits=d_logits.reshape(b, steps, V).transpose(1, 0, 2).reshape(-1), dctc=d_ctc,
                          ctc_logits=ctc_logits.reshape(-1))
        # backward
        d_enc = self.attn_bwd(d_logits, atr)
        dct = d_ctc.reshape(b * t, V)
        self.g["ctc.w"] += dot64(dct.T, enc.reshape(b * t, H))
        self.g["ctc.b"] += sum64(dct, axis=0)
        d_enc = (d_enc + dot64(dct, self.p["ctc.w"]).reshape(-1)).astype(F32)
        d = d_enc
        self.debug["d_enc"] = d_enc
        for li in range(cfg.rnn_layers - 1, -1, -1):
            d = self.bilstm_layer_bwd(li, d, rtr[li])
        self.debug["dfeat"] = d
        self.cnn_bwd(np.ascontiguousarray(d.astype(F32)), ctr)
        if optimize:
            self.optimizer_step()
        return dict(loss=total, attn=attn_loss, ctc=ctc_loss)

    # -- clip + Muon/Adam + requantize: src/main.rs:2373-2410, src/opt.rs ----
    def optimizer_step(self):
        cfg = self.cfg
        lr, wd = F32(cfg.lr), F32(cfg.weight_decay)
        kinds = {n: k for n, _, k in manifest(cfg)}
        if self.t < cfg.clip_warmup:
            sq = sum(float((g.astype(np.float64) ** 2).sum()) for g in self.g.values())
            norm = math.sqrt(sq)
            f = F32(5.0 / (norm + 1e-6)) if norm > 5.0 else F32(1.0)
        else:
            f = F32(1.0)
        self.t += 1
        bc1, bc2 = bias_corrections(self.t)
        for n, k in kinds.items():
            if k == "conv_w":
                continue
            g = self.g[n] if not f < 1.0 else (self.g[n] * f).astype(F32)
            p = self.p[n]
            if k == "vec":
                m = self.adam_m.setdefault(n, np.zeros_like(p))
                v = self.adam_v.setdefault(n, np.zeros_like(p))
                adam_vec_step(p, g, m, v, lr, wd, bc1, bc2)
            else:
                muon_host_step(p, g, lr, wd, cfg.muon_cap)
        for c in conv_specs(cfg):  # device Muon per conv (src/qnet.rs:559-573)
            w, g = self.p[f"{c.name}.w"], self.g[f"{c.name}.w"]
            gsq = np.zeros(1, np.float64)
            self.be("launch_sum_sq_add_f32", g, gsq, g.size)
            self.be("launch_muon_step_f32", w, g, gsq, w.size, float(lr), float(wd), float(f),
                    float(min(c.cout, c.k)), float(max(c.cout, c.k)), float(cfg.muon_cap), 1)
        for cs in self.convs.values():
            self.requantize(cs)
