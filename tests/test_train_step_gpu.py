"""Parity of the fused device-resident QAT training step against the CPU
oracle of the reference's step (oracle/step_oracle.py driving the
reference's own CPU backend where it was built, else our C restatement).

Same injected weights, same batch; compared after one step:
  * losses (total, attention CE, CTC): rel 1e-4;
  * every parameter's gradient: max |g_gpu - g_ref| <= 2e-3 * max |g_ref| (+1e-7);
  * every parameter after the clip + Muon/Adam step: max |p_gpu - p_ref|
    <= 1e-4 * max |p_ref| (+1e-7).
The integer path (im2col, int8 GEMMs, quantisers) is bit-exact; the
tolerances absorb float summation order in BN statistics, the LSTM /
attention products and the rare int8 rounding flip a 1-ulp difference
causes downstream (the same bound the reference's own tests allow: 1e-3
relative for gradients).
"""
import sys

import numpy as np
import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))
import step_oracle as so  # noqa: E402

pytestmark = pytest.mark.gpu


def _setup(geom, B, seed, wgrad_mode=0):
    import trba_b200.model as tm
    ocfg = so.Config(**geom, wgrad_mode="compat" if wgrad_mode == 0 else "correct")
    params = so.init_params(ocfg, seed)
    gm = tm.QatModel(tm.Config(**geom, batch=B, wgrad_mode=wgrad_mode))
    man = gm.manifest()
    onames = [n for n, _, _ in so.manifest(ocfg)]
    assert [e[0] for e in man] == onames, "parameter manifest differs from the reference order"
    flat = np.concatenate([params[n].ravel() for n in onames]).astype(np.float32)
    assert flat.size == gm.n_params
    gm.set_params(flat)
    return ocfg, params, gm, man


def _to_dev(img, ti, tg, ct, steps):
    import torch
    import trba_b200.model as tm
    ti32, tg32, ctc, lens = tm.pack_labels(ti, tg, ct, steps)
    d = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (img, ti32, tg32, ctc, lens)]
    return d


def _compare(man, got_flat, want: dict, rel, what):
    worst = []
    for name, off, rows, cols, kind in man:
        n = rows * cols if cols else rows
        g = got_flat[off:off + n].astype(np.float64)
        w = want[name].ravel().astype(np.float64)
        d = float(np.abs(g - w).max())
        scale = float(np.abs(w).max())
        worst.append((d / (scale + 1e-30), name, d, scale))
        if not d <= rel * scale + 1e-7:
            bad = sorted(worst, reverse=True)[:5]
            raise AssertionError(f"{what} of {name}: max diff {d:.3g} vs scale {scale:.3g}; worst: {bad}")
    return sorted(worst, reverse=True)[:3]


@pytest.mark.parametrize("geom,B", [
    (dict(img_w=64, max_len=4), 8),       # TRBA-small 32x64 (the reference's CPU-runnable case)
    (dict(img_w=160, max_len=20), 4),     # 32x160, max_len 20
], ids=["32x64_b8", "32x160_b4"])
@pytest.mark.parametrize("wgrad_mode", [0, 1], ids=["compat", "correct"])
def test_train_step_matches_oracle(geom, B, wgrad_mode, lib, cuda):
    ocfg, params, gm, man = _setup(geom, B, seed=1234, wgrad_mode=wgrad_mode)
    img, ti, tg, ct = so.make_batch(ocfg, B, seed=99)
    orc = so.OracleTrba(ocfg, params)
    res = orc.train_step(img, ti, tg, ct)
    dev = _to_dev(img, ti, tg, ct, ocfg.steps)
    gm.forward_backward(*dev)
    loss = gm.loss()
    want = np.array([res["loss"], res["attn"], res["ctc"]])
    assert np.allclose(loss, want, rtol=1e-4, atol=1e-6), (loss, want)
    _compare(man, gm.get_grads(), orc.g, 2e-3, "gradient")
    gm.optimizer_step()
    _compare(man, gm.get_params(), orc.p, 1e-4, "updated parameter")
    assert lib.trba_tc_error_poll(1) == 0
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


def test_running_stats_follow_the_batch_statistics(lib, cuda):
    geom = dict(img_w=64, max_len=4)
    ocfg, params, gm, man = _setup(geom, 8, seed=5)
    img, ti, tg, ct = so.make_batch(ocfg, 8, seed=7)
    orc = so.OracleTrba(ocfg, params)
    orc.train_step(img, ti, tg, ct)
    gm.forward_backward(*_to_dev(img, ti, tg, ct, ocfg.steps))
    got = gm.running_stats()
    want = np.concatenate([np.concatenate([orc.run_mean[c.name], orc.run_var[c.name]]) for c in so.conv_specs(ocfg)])
    assert np.allclose(got, want, rtol=1e-4, atol=1e-5)


def test_host_entry_point_equals_device_entry_point(lib, cuda):
    import trba_b200.model as tm
    geom = dict(img_w=64, max_len=4)
    ocfg, params, gm, man = _setup(geom, 8, seed=3)
    _, _, gm2, _ = _setup(geom, 8, seed=3)
    img, ti, tg, ct = so.make_batch(ocfg, 8, seed=11)
    dev = _to_dev(img, ti, tg, ct, ocfg.steps)
    gm.train_step(*dev)
    l1 = gm.loss()
    ti32, tg32, ctc, lens = tm.pack_labels(ti, tg, ct, ocfg.steps)
    l2 = gm2.train_step_host(np.ascontiguousarray(img), ti32, tg32, ctc, lens)
    assert np.array_equal(l1, l2)
    assert np.array_equal(gm.get_params(), gm2.get_params())
