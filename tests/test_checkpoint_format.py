"""The checkpoint byte layout (trba_b200.checkpoint) on CPU, through a model
stand-in: write V6, parse it back field by field, and the layout the
reference's reader expects (magic, meta, geometry, named tensors with their
Adam moments, BN statistics per conv)."""
import struct

import numpy as np

import trba_b200.checkpoint as ck


class FakeModel:
    class cfg:
        img_h, img_w, max_len, hidden, classes, rnn_layers, fd = 32, 64, 4, 64, 130, 2, 128

    def __init__(self):
        self._man = [("stem.0.w", 0, 4, 3, 0), ("stem.0.gamma", 12, 4, 0, 2), ("stem.0.beta", 16, 4, 0, 2),
                     ("attn.gen.w", 20, 2, 5, 1)]
        self.n_params = 30
        self.p = np.arange(30, dtype=np.float32) * 0.5
        self.m = np.linspace(0, 1, 30, dtype=np.float32)
        self.v = np.linspace(1, 2, 30, dtype=np.float32)
        self.rs = np.arange(8, dtype=np.float32)
        self.t = 7

    def manifest(self):
        return self._man

    def get_params(self):
        return self.p.copy()

    def get_moments(self, m, v):
        m[:] = self.m
        v[:] = self.v

    def running_stats(self):
        return self.rs.copy()

    def step_count(self):
        return self.t

    def conv_channels(self):
        return [4]

    def set_params(self, p):
        self.p = p.copy()
        self.m[:] = 0
        self.v[:] = 0
        self.t = 0

    def set_moments(self, m, v):
        self.m, self.v = m.copy(), v.copy()

    def set_running_stats(self, rs):
        self.rs = rs.copy()

    def set_step_count(self, t):
        self.t = t


def test_v6_layout_and_round_trip(tmp_path):
    src = FakeModel()
    path = tmp_path / "x.ckpt"
    ck.save(src, path, epoch_done=2, batch_in_epoch=5)
    raw = path.read_bytes()
    assert raw[:8] == b"TRBA_V6\n"
    head = struct.unpack("<11Q", raw[8:8 + 88])
    assert head[:3] == (2, 5, 7) and head[3:10] == (32, 64, 4, 64, 130, 2, 128) and head[10] == 4
    name_len = struct.unpack("<Q", raw[96:104])[0]
    assert raw[104:104 + name_len] == b"stem.0.w"
    parsed = ck.read(path)
    assert [p[0] for p in parsed["params"]] == ["stem.0.w", "stem.0.gamma", "stem.0.beta", "attn.gen.w"]
    # Adam moments only on vectors (kind 2); empty elsewhere
    assert [p[2].size for p in parsed["params"]] == [0, 4, 4, 0]
    assert np.array_equal(parsed["params"][1][2], src.m[12:16])
    assert len(parsed["convs"]) == 1 and np.array_equal(parsed["convs"][0][1], src.rs[4:8])
    dst = FakeModel()
    dst.p[:] = -1
    meta = ck.load(dst, path)
    assert meta["opt_t"] == 7 and meta["epoch_done"] == 2
    assert np.array_equal(dst.p, src.p) and np.array_equal(dst.rs, src.rs) and dst.t == 7
    assert np.array_equal(dst.m[12:20], src.m[12:20]) and not dst.m[:12].any()


def test_geometry_mismatch_is_refused(tmp_path):
    src = FakeModel()
    path = tmp_path / "x.ckpt"
    ck.save(src, path)
    dst = FakeModel()
    dst.cfg = type("cfg", (), dict(img_h=32, img_w=160, max_len=20, hidden=64, classes=130, rnn_layers=2, fd=128))
    try:
        ck.load(dst, path)
    except ValueError as e:
        assert "geometry" in str(e)
    else:
        raise AssertionError("a checkpoint of another geometry loaded")
