"""The halo tiling of the tensor-core input gradient, checked on the CPU.

The library's own host-side planner (trba_tc_dgrad_plan: the halo geometry,
stride-phase classes, tile counts, stage sizes and per-tap offsets the kernel
is launched with) is
combined with a numpy restatement of what the kernels do with it:
split_halo_kernel's padded plane layout and exact three-term split,
image_element's weight blocks, the halo producer's bulk copies (one per
plane and 8-channel slab: R rows from plane row tile * 128 * mb), the MMA
warp's shifted 128-row windows and the epilogue's position -> pixel map.
Every copy and window is asserted to stay inside its buffer, the sizes the
launch asks for inside the B200's limits, and the result must equal the
oracle's launch_conv_backward_grad_input_i8 on the same inputs (f64
accumulation here: within 1e-5 of the gradient's scale).  No GPU."""
import ctypes as C

import numpy as np
import pytest

A16 = lambda x: (x + 15) & ~15  # noqa: E731
FIELDS = ("halo BN Npad ntn tiles taps KC nchunks mb R sa sb Hq Wq dmin mpos rows plane_elems img_bytes smem "
          "tmem").split()
SMEM_LIMIT = 232448  # dynamic shared memory per CTA (opt-in) on sm_100a


def _plan(lib, *shape):
    out = (C.c_longlong * 400)()
    n = lib.trba_tc_dgrad_plan(*[C.c_int(x) for x in shape], out, 400)
    if n < 0:
        return None
    f = list(out[:n])
    p = dict(zip(FIELDS, f[:21]))
    p["classes"] = []
    if p["halo"]:
        i = 22
        for _ in range(f[21]):
            cl = dict(zip("py px Hc Wc ntaps tile0 mtiles b_off".split(), f[i:i + 8]))
            i += 8
            cl["taps"] = [tuple(f[i + 3 * t:i + 3 * t + 3]) for t in range(cl["ntaps"])]
            i += 3 * cl["ntaps"]
            p["classes"].append(cl)
        assert i == n
    return p


def _split(v):
    """split_pair: hi / mid / lo bf16 terms (as f32) whose sum is exactly v."""
    u = v.view(np.uint32)
    hi = (u & 0xFFFF0000).view(np.float32)
    r = (v - hi).astype(np.float32)
    mid = (r.view(np.uint32) & 0xFFFF0000).view(np.float32)
    lo = (r - mid).astype(np.float32)
    assert ((lo.view(np.uint32) & 0xFFFF) == 0).all(), "lo term not representable in bf16"
    return hi, mid, lo


def _emulate(p, dy, wq, wld, w_s, B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo):
    BN, KC, mb, R, Hq, Wq, dmin = p["BN"], p["KC"], p["mb"], p["R"], p["Hq"], p["Wq"], p["dmin"]
    rows, mpos, ntn, nch = p["rows"], p["mpos"], p["ntn"], p["nchunks"]
    nsl, MT = KC // 8, 128 * mb
    assert p["plane_elems"] == cout * rows
    # split_halo_kernel: planes[term][slab][row][8]
    planes = np.zeros((3, cout // 8, rows, 8), np.float32)
    pos = np.arange(rows) + dmin
    ok = (pos >= 0) & (pos < mpos)
    b_ = np.where(ok, pos // (Hq * Wq), 0)
    rem = np.where(ok, pos - b_ * Hq * Wq, 0)
    yy, xx = rem // Wq, rem % Wq
    real = ok & (yy < ho) & (xx < wo)
    vals = np.zeros((rows, cout), np.float32)
    vals[real] = dy[b_[real], :, yy[real], xx[real]]
    for t, term in enumerate(_split(vals)):
        planes[t] = term.reshape(rows, cout // 8, 8).transpose(1, 0, 2)
    # image_element: blocks (class, N tile, chunk, tap) of [KC / 8][BN][8]
    nblocks = sum(ntn * nch * cl["ntaps"] for cl in p["classes"])
    img = np.zeros((nblocks, nsl, BN, 8), np.float32)
    for cl in p["classes"]:
        for nt in range(ntn):
            for c in range(nch):
                for t, (tkh, tkw, _) in enumerate(cl["taps"]):
                    blk = cl["b_off"] + (nt * nch + c) * cl["ntaps"] + t
                    for s in range(nsl):
                        for j in range(8):
                            co = c * KC + s * 8 + j
                            ci = nt * BN + np.arange(BN)
                            m = ci < cin
                            img[blk, s, m, j] = wq[co, ci[m] * kh * kw + tkh * kw + tkw]
    assert img.size * 2 == p["img_bytes"]
    gi = np.full((B, cin, h, w), np.nan, np.float64)
    for tile in range(p["tiles"]):
        cl = [c for c in p["classes"] if c["tile0"] <= tile][-1]
        local = tile - cl["tile0"]
        assert local < cl["mtiles"] * ntn
        mt, nt = divmod(local, ntn)
        row0 = mt * MT
        acc = np.zeros((MT, BN), np.float64)
        for c in range(nch if cl["ntaps"] else 0):
            # halo producer: one bulk copy of R rows per (term, slab)
            assert 0 <= row0 and row0 + R <= rows, "halo copy past the plane"
            halo = planes[:, c * nsl:(c + 1) * nsl, row0:row0 + R, :]           # [3][nsl][R][8]
            a = halo.transpose(0, 2, 1, 3).reshape(3, R, KC).astype(np.float64)  # K index s * 8 + j
            for t, (_, _, off) in enumerate(cl["taps"]):
                blk = cl["b_off"] + (nt * nch + c) * cl["ntaps"] + t
                assert blk < nblocks
                bk = img[blk].transpose(1, 0, 2).reshape(BN, KC).astype(np.float64)
                for i in range(mb):
                    lo_, hi_ = off + i * 128, off + i * 128 + 128
                    assert 0 <= lo_ and hi_ <= R, "MMA window outside the halo"
                    for term in range(3):
                        acc[i * 128:(i + 1) * 128] += a[term, lo_:hi_] @ bk.T
        # epilogue: class position (b, i, j) -> pixel (py + sh i, px + sw j)
        P = mt * MT + np.arange(MT)
        bb, rr = P // (Hq * Wq), P % (Hq * Wq)
        ci_, cj_ = rr // Wq, rr % Wq
        rv = (P < mpos) & (ci_ < cl["Hc"]) & (cj_ < cl["Wc"])
        y, x = cl["py"] + sh * ci_, cl["px"] + sw * cj_
        n0 = nt * BN
        ncols = min(BN, cin - n0)
        for m in np.nonzero(rv)[0]:
            assert np.isnan(gi[bb[m], n0, y[m], x[m]]), "pixel written twice"
            gi[bb[m], n0:n0 + ncols, y[m], x[m]] = acc[m, :ncols] * w_s
    return gi


# (B, Cin, H, W, Cout, kh, kw, sh, sw, ph, pw): the model's convs (small
# batches) and odd ones (padded N, two N tiles, a 1x1 conv, asymmetric
# kernels, padding and strides, odd planes, phases without taps)
SHAPES = [
    (1, 16, 32, 160, 32, 3, 3, 1, 1, 1, 1),   # stem.3
    (2, 32, 16, 80, 64, 3, 3, 2, 2, 1, 1),    # layer1.0.conv1 (stride 2)
    (2, 32, 16, 80, 64, 1, 1, 2, 2, 0, 0),    # layer1.0.downsample (three phases without taps)
    (2, 64, 8, 40, 64, 3, 3, 1, 1, 1, 1),     # layer2.x
    (2, 64, 8, 40, 128, 3, 3, 2, 2, 1, 1),    # layer3.0.conv1
    (3, 128, 4, 20, 128, 3, 3, 1, 1, 1, 1),   # layer3 / layer4
    (3, 128, 4, 20, 128, 2, 2, 2, 1, 0, 1),   # conv_out.0 (stride (2, 1), pad (0, 1))
    (3, 128, 2, 21, 128, 2, 2, 1, 1, 0, 0),   # conv_out.3
    (3, 24, 7, 9, 16, 3, 3, 1, 1, 1, 1),      # Cin 24: padded N
    (1, 200, 4, 4, 16, 3, 3, 1, 1, 1, 1),     # two N tiles
    (2, 16, 5, 7, 32, 1, 1, 1, 1, 0, 0),      # 1x1
    (2, 8, 6, 5, 16, 3, 2, 1, 1, 1, 0),       # asymmetric kernel and padding
    (2, 8, 6, 9, 16, 3, 3, 1, 1, 0, 2),       # padding 0 on one axis, 2 on the other
    (2, 8, 7, 9, 16, 3, 3, 2, 2, 1, 1),       # odd planes, stride 2: classes of different sizes
    (2, 24, 9, 6, 32, 3, 3, 2, 1, 1, 1),      # stride (2, 1)
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "b{}_c{}_{}x{}_o{}_k{}x{}_s{}{}".format(*s[:9]))
@pytest.mark.parametrize("tiling", [(0, 0), (1, 16), (2, 32), (3, 32), (4, 16), (1, 64)],
                         ids=["auto", "mb1_kc16", "mb2_kc32", "mb3_kc32", "mb4_kc16", "mb1_kc64"])
def test_halo_plan_matches_oracle(shape, tiling, lib, oracle):
    B, cin, h, w, cout, kh, kw, sh, sw, ph, pw = shape
    ho, wo = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
    lib.trba_tc_dgrad_tiling(*tiling)
    try:
        p = _plan(lib, B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo)
    finally:
        lib.trba_tc_dgrad_tiling(0, 0)
    assert p is not None
    if not p["halo"]:
        assert tiling != (0, 0), "conv left on the class tiling"
        pytest.skip("forced tile does not fit this conv")
    assert p["smem"] <= SMEM_LIMIT and p["tmem"] <= 512 and p["R"] * 16 < (1 << 18)
    assert p["sa"] in (1, 2) and 2 <= p["sb"] <= 16
    rng = np.random.default_rng(sum(shape))
    dy = (rng.standard_normal((B, cout, ho, wo)) * 1e-3).astype(np.float32)
    dy[rng.random(dy.shape) < 0.3] = 0.0
    k = cin * kh * kw
    wld = A16(k)
    wq = np.zeros((A16(cout), wld), np.int8)
    wq[:cout, :k] = rng.integers(-127, 128, (cout, k))
    w_s = 0.0123
    want = np.zeros(B * cin * h * w, np.float32)
    oracle.launch_conv_backward_grad_input_i8(dy.ctypes.data, wq.ctypes.data, wld, w_s, want.ctypes.data, B, cin,
                                              h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo, None)
    got = _emulate(p, dy, wq, wld, w_s, B, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo)
    assert not np.isnan(got).any(), "pixels never written"
    scale = float(np.abs(want).max())
    err = float(np.abs(got.ravel() - want).max())
    assert err <= 1e-5 * scale, f"max diff {err:.3g} vs scale {scale:.3g}"


def test_model_convs_get_the_halo_tiling(lib):
    """Every conv of the 32x160 model at batch 512 whose input gradient is
    computed (all but the first) is on the halo tiling, strided ones included;
    the override -1 keeps them on the class tiling."""
    convs = [(16, 32, 160, 32, 3, 3, 1, 1, 1, 1), (32, 16, 80, 64, 3, 3, 2, 2, 1, 1),
             (32, 16, 80, 64, 1, 1, 2, 2, 0, 0), (64, 8, 40, 64, 3, 3, 1, 1, 1, 1),
             (64, 8, 40, 128, 3, 3, 2, 2, 1, 1), (64, 8, 40, 128, 1, 1, 2, 2, 0, 0),
             (128, 4, 20, 128, 3, 3, 1, 1, 1, 1), (128, 4, 20, 128, 2, 2, 2, 1, 0, 1),
             (128, 2, 21, 128, 2, 2, 1, 1, 0, 0)]
    for cin, h, w, cout, kh, kw, sh, sw, ph, pw in convs:
        ho, wo = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
        p = _plan(lib, 512, cin, h, w, cout, kh, kw, sh, sw, ph, pw, ho, wo)
        assert p["halo"] == 1, (cin, h, w, sh)
    lib.trba_tc_dgrad_tiling(-1, 0)
    try:
        p = _plan(lib, 512, 128, 4, 20, 128, 3, 3, 1, 1, 1, 1, 4, 20)
    finally:
        lib.trba_tc_dgrad_tiling(0, 0)
    assert p["halo"] == 0
