"""Synthetic inputs and seeded weights for the QAT training step.

The reference trains on handwriting line images and initialises with
rand::thread_rng (not seedable); benchmarks and tests here use:

  * weights: Glorot-uniform with the reference's limits (src/qnet.rs:483,
    src/rnn.rs:28-29,84, src/attn.rs:53-78, LinearF src/qnet.rs:109), BN
    gamma 1 / beta 0, biases 0, drawn from numpy's PCG64 with a seed;
  * images: pixels uniform in [0, 1], quantised like src/main.rs:881
    (round((p*2-1)*127) clamped to +-127, scale 1/127), NCHW int8;
  * labels: lengths from a log-normal with the corpus quantiles the
    reference documents (median 5, p90 11), clipped to [1, max_len]; tokens
    uniform in [3, classes); teacher-forcing input / target / CTC target
    built as src/main.rs:2063-2109 does.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
LEN_P50, LEN_P90 = 5, 11


def glorot_limit(name: str, rows: int, cols: int, kind: int, cfg, conv_k: dict) -> float:
    H, V = cfg.hidden, cfg.classes
    if kind == 0:  # conv: sqrt(6 / (cin*kh*kw + cout*kh*kw))
        k, khw = conv_k[name]
        return math.sqrt(6.0 / (k + rows * khw))
    if name.startswith("rnn") and name.endswith(".w_ih"):
        return math.sqrt(6.0 / (cols + 4 * H))
    if name.startswith("rnn") and name.endswith(".w_hh"):
        return math.sqrt(6.0 / (H + 4 * H))
    if name == "attn.w_ih":
        return math.sqrt(6.0 / (H + V + 4 * H))
    if name == "attn.w_hh":
        return math.sqrt(6.0 / (H + 4 * H))
    return math.sqrt(6.0 / (rows + cols))


def conv_geometry(cfg) -> dict:
    """name.w -> (K = cin*kh*kw, kh*kw) of every conv (src/qnet.rs:1435-1455)."""
    fd = cfg.fd
    w = [fd // 8, fd // 4, fd // 2, fd // 2, fd, fd]
    out = {"stem.0.w": (3 * 9, 9), "stem.3.w": (w[0] * 9, 9)}
    blocks = [("layer1.0", w[1], w[2], 2), ("layer2.0", w[2], w[3], 1), ("layer2.1", w[3], w[3], 1),
              ("layer3.0", w[3], w[4], 2)] + [(f"layer3.{i}", w[4], w[4], 1) for i in range(1, 5)] + \
             [(f"layer4.{i}", w[5], w[5], 1) for i in range(3)]
    for name, ic, oc, s in blocks:
        if s != 1 or ic != oc:
            out[f"{name}.downsample.0.w"] = (ic, 1)
        out[f"{name}.conv1.w"] = (ic * 9, 9)
        out[f"{name}.conv2.w"] = (oc * 9, 9)
    out["conv_out.0.w"] = (w[5] * 4, 4)
    out["conv_out.3.w"] = (w[5] * 4, 4)
    return out


def init_params(manifest, cfg, seed: int) -> np.ndarray:
    """Flat fp32 parameter vector in manifest order ([(name, off, rows, cols, kind)])."""
    rng = np.random.default_rng(seed)
    ck = conv_geometry(cfg)
    n = max(off + (r * c if c else r) for _, off, r, c, _ in manifest)
    flat = np.zeros(n, F32)
    for name, off, rows, cols, kind in manifest:
        size = rows * cols if cols else rows
        if kind == 2:
            flat[off:off + size] = 1.0 if name.endswith(".gamma") else 0.0
        else:
            lim = glorot_limit(name, rows, cols, kind, cfg, ck)
            flat[off:off + size] = rng.uniform(-lim, lim, size=size).astype(F32)
    return flat


def quantise_image(pix: np.ndarray) -> np.ndarray:
    v = (pix.astype(F32) * F32(2.0) - F32(1.0)) * F32(127.0)
    r = np.sign(v) * np.floor(np.abs(v) + F32(0.5))  # round half away from zero
    return np.clip(r, -127, 127).astype(np.int8)


def sample_lengths(rng, b: int, max_len: int) -> np.ndarray:
    mu = math.log(LEN_P50)
    sigma = (math.log(LEN_P90) - mu) / 1.2815515655446004
    l = np.rint(np.exp(rng.normal(mu, sigma, size=b))).astype(np.int64)
    return np.clip(l, 1, max_len)


def make_batch(cfg, b: int, seed: int, fixed_len: int | None = None):
    """(img [B,3,H,W] int8, text_in [B,S], target [B,S], ctc [B,S] (-1 pad),
    ctc_len [B]) as int32 arrays, S = max_len + 1."""
    rng = np.random.default_rng(seed)
    img = quantise_image(rng.random((b, 3, cfg.img_h, cfg.img_w), dtype=np.float32))
    lens = np.full(b, fixed_len) if fixed_len else sample_lengths(rng, b, cfg.max_len)
    S = cfg.max_len + 1
    text_in = np.full((b, S), cfg.pad, np.int32)
    target = np.full((b, S), cfg.pad, np.int32)
    ctc = np.full((b, S), -1, np.int32)
    ctc_len = np.zeros(b, np.int32)
    for i in range(b):
        l = int(min(lens[i], cfg.max_len))
        toks = rng.integers(3, cfg.classes, size=l)
        text_in[i, 0] = cfg.sos
        text_in[i, 1:1 + l] = toks
        target[i, :l] = toks
        target[i, l] = cfg.eos
        ctc[i, :l] = toks
        ctc[i, l] = cfg.eos
        ctc_len[i] = l + 1
    return img, text_in, target, ctc, ctc_len
