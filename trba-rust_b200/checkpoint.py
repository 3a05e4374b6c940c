"""The reference's checkpoint files (later snapshot src/main.rs:1099-1338):
TRBA_V6 written, TRBA_V6 / V5 / V4 read, so weights trained here load in the
reference's trainer and the reference's checkpoints resume here.

Layout (little-endian u64 counts, f32 data; "f32s" = u64 length + data):

    magic            b"TRBA_V6\\n" | b"TRBA_V5\\n" | b"TRBA_V4\\n"
    epoch_done       u64
    batch_in_epoch   u64                       (V5, V6)
    opt_t            u64
    geometry         7 x u64: img_h img_w max_len hidden classes rnn_layers
                     feat_dim                   (V6)
    n_params         u64
    per parameter, in Model::params() order:
      name           u64 length + bytes         (V6)
      value          f32s
      adam m, v      f32s each, empty when the parameter has no Adam state (V5, V6)
    per conv layer, in SEResNetQ::convs_mut() order:
      run_mean, run_var   f32s each
      conv moments m, v   f32s each (V5, V6; empty: the conv Muon keeps none)

Loading requires the model's geometry (shapes in manifest order); the
reference's shape surgery into another geometry is not restated.  Adam
moments are restored only for parameters whose saved moments have the
parameter's length (the reference's rule), and only when the file's
geometry equals the model's.
"""
from __future__ import annotations

import os
import struct
from pathlib import Path

import numpy as np

MAGIC_V6 = b"TRBA_V6\n"
MAGIC_V5 = b"TRBA_V5\n"
MAGIC_V4 = b"TRBA_V4\n"

KIND_VECTOR = 2  # manifest kind of Adam-managed parameters


def _u64(f, v: int):
    f.write(struct.pack("<Q", int(v)))


def _f32s(f, a):
    a = np.ascontiguousarray(a, dtype="<f4").ravel()
    _u64(f, a.size)
    f.write(a.tobytes())


def _read_u64(f) -> int:
    b = f.read(8)
    if len(b) != 8:
        raise ValueError("checkpoint truncated")
    return struct.unpack("<Q", b)[0]


def _read_f32s(f) -> np.ndarray:
    n = _read_u64(f)
    b = f.read(4 * n)
    if len(b) != 4 * n:
        raise ValueError("checkpoint truncated")
    return np.frombuffer(b, dtype="<f4").astype(np.float32)


def geometry(model) -> tuple:
    c = model.cfg
    return (c.img_h, c.img_w, c.max_len, c.hidden, c.classes, c.rnn_layers, c.fd)


def save(model, path: str | os.PathLike, epoch_done: int = 0, batch_in_epoch: int = 0):
    """Writes a TRBA_V6 checkpoint of `model` (a trba_b200.model.QatModel):
    parameters, Adam moments, BN running statistics, the optimiser step.
    Written to path + ".tmp" and renamed, as the reference does."""
    path = Path(path)
    man = model.manifest()
    p = model.get_params()
    n = model.n_params
    m_all = np.empty(n, np.float32)
    v_all = np.empty(n, np.float32)
    model.get_moments(m_all, v_all)
    rs = model.running_stats()
    t = model.step_count()
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "wb") as f:
        f.write(MAGIC_V6)
        _u64(f, epoch_done)
        _u64(f, batch_in_epoch)
        _u64(f, t)
        for g in geometry(model):
            _u64(f, g)
        _u64(f, len(man))
        for name, off, rows, cols, kind in man:
            size = rows * cols if cols else rows
            nb = name.encode()
            _u64(f, len(nb))
            f.write(nb)
            _f32s(f, p[off:off + size])
            if kind == KIND_VECTOR and t > 0:
                _f32s(f, m_all[off:off + size])
                _f32s(f, v_all[off:off + size])
            else:
                _f32s(f, np.zeros(0, np.float32))
                _f32s(f, np.zeros(0, np.float32))
        o = 0
        for cout in model.conv_channels():
            _f32s(f, rs[o:o + cout])
            _f32s(f, rs[o + cout:o + 2 * cout])
            _f32s(f, np.zeros(0, np.float32))
            _f32s(f, np.zeros(0, np.float32))
            o += 2 * cout
    os.replace(tmp, path)


def read(path: str | os.PathLike) -> dict:
    """Parses a TRBA_V6 / V5 / V4 file into a dict: version, epoch_done,
    batch_in_epoch, opt_t, geometry (V6 only, else None), params [(name or
    None, value, m, v)], convs [(run_mean, run_var, m, v)]."""
    with open(path, "rb") as f:
        magic = f.read(8)
        if magic == MAGIC_V6:
            version, v5, v6 = 6, True, True
        elif magic == MAGIC_V5:
            version, v5, v6 = 5, True, False
        elif magic == MAGIC_V4:
            version, v5, v6 = 4, False, False
        else:
            raise ValueError(f"bad checkpoint magic {magic!r}")
        out = {"version": version, "epoch_done": _read_u64(f)}
        out["batch_in_epoch"] = _read_u64(f) if v5 else 0
        out["opt_t"] = _read_u64(f)
        out["geometry"] = tuple(_read_u64(f) for _ in range(7)) if v6 else None
        params = []
        for _ in range(_read_u64(f)):
            name = f.read(_read_u64(f)).decode() if v6 else None
            val = _read_f32s(f)
            m = _read_f32s(f) if v5 else np.zeros(0, np.float32)
            v = _read_f32s(f) if v5 else np.zeros(0, np.float32)
            params.append((name, val, m, v))
        convs = []
        while True:
            head = f.read(8)
            if not head:
                break
            f.seek(-8, 1)
            rm, rv = _read_f32s(f), _read_f32s(f)
            cm = _read_f32s(f) if v5 else np.zeros(0, np.float32)
            cv = _read_f32s(f) if v5 else np.zeros(0, np.float32)
            convs.append((rm, rv, cm, cv))
        out["params"], out["convs"] = params, convs
    return out


def load(model, path: str | os.PathLike) -> dict:
    """Loads a TRBA_V6 / V5 / V4 checkpoint into `model`: parameters (by name
    in V6, by manifest position in V5 / V4), BN running statistics, the
    optimiser step and the Adam moments of every tensor whose saved moments
    have the parameter's length.  A V6 file of another geometry is refused;
    V5 files carry no geometry (their moments load whenever the lengths
    match) and V4 files no moments.  Returns the file's meta data."""
    ck = read(path)
    man = model.manifest()
    if ck["geometry"] is not None and tuple(ck["geometry"]) != geometry(model):
        raise ValueError(f"checkpoint geometry {ck['geometry']} differs from the model's {geometry(model)}; "
                         "shape surgery into another geometry is not supported")
    if len(ck["params"]) != len(man):
        raise ValueError(f"checkpoint has {len(ck['params'])} tensors, the model {len(man)}")
    by_name = {e[0]: e for e in man}
    n = model.n_params
    flat = model.get_params()
    m_all = np.zeros(n, np.float32)
    v_all = np.zeros(n, np.float32)
    for i, (name, val, m, v) in enumerate(ck["params"]):
        e = by_name.get(name) if name is not None else man[i]
        if e is None:
            raise ValueError(f"checkpoint tensor {name} is not a parameter of the model")
        _, off, rows, cols, _ = e
        size = rows * cols if cols else rows
        if val.size != size:
            raise ValueError(f"{e[0]}: {val.size} values in the checkpoint, {size} in the model")
        flat[off:off + size] = val
        if m.size == size and v.size == size:
            m_all[off:off + size] = m
            v_all[off:off + size] = v
    chans = model.conv_channels()
    if len(ck["convs"]) != len(chans):
        raise ValueError(f"checkpoint has BN statistics of {len(ck['convs'])} convolutions, the model {len(chans)}")
    rs = np.empty(2 * sum(chans), np.float32)
    o = 0
    for (rm, rv, _, _), cout in zip(ck["convs"], chans):
        if rm.size != cout or rv.size != cout:
            raise ValueError("BN running statistics: channel count differs")
        rs[o:o + cout], rs[o + cout:o + 2 * cout] = rm, rv
        o += 2 * cout
    model.set_params(flat)  # resets moments, step and re-quantises
    model.set_running_stats(rs)
    model.set_moments(m_all, v_all)
    model.set_step_count(ck["opt_t"])
    return {k: ck[k] for k in ("version", "epoch_done", "batch_in_epoch", "opt_t", "geometry")}
