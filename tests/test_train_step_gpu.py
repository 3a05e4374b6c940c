"""Parity of the fused device-resident QAT training step against the CPU
oracle of the reference's step (oracle/step_oracle.py driving
oracle/liboracle.so, our C restatement of the reference's CPU backend, which
tests/test_oracle_golden.py pins to the reference's own backend).

Same injected weights, same batch.  Every integer / quantisation operation
is exact on both sides, every float reduction is accumulated in f64 and
rounded once on both sides, and transcendentals are correctly rounded on
both sides, so one step is compared bit for bit:
  * the three losses and the intermediate tensors (features, encoder output,
    logits, their gradients): identical;
  * every parameter gradient: identical (max |diff| <= 1e-6 * max |g| is
    allowed for a rounding tie in an f64 -> f32 conversion);
  * every parameter after clip + Muon/Adam + re-quantisation: max |diff|
    <= 1e-6 * max |p| (f64 sums of the per-conv gradient norms are combined
    in a different order).
Over 200 steps the loss curves must stay within 1% of each other (the bar
the reference's behaviour is held to); in practice they coincide.
"""
import sys

import numpy as np
import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))
import step_oracle as so  # noqa: E402

pytestmark = pytest.mark.gpu


def _oracle_backend():
    """The deterministic C restatement (single f64 sums in BN statistics);
    tests/test_oracle_golden.py pins it to the reference's CPU backend."""
    return so.CpuBackend(REPO / "oracle" / "liboracle.so")


def _setup(geom, B, seed, wgrad_mode=0, dgrad_mode=0):
    import trba_b200.model as tm
    ocfg = so.Config(**geom, wgrad_mode="compat" if wgrad_mode == 0 else "correct")
    params = so.init_params(ocfg, seed)
    gm = tm.QatModel(tm.Config(**geom, batch=B, wgrad_mode=wgrad_mode, dgrad_mode=dgrad_mode))
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
    orc = so.OracleTrba(ocfg, params, _oracle_backend())
    res = orc.train_step(img, ti, tg, ct)
    dev = _to_dev(img, ti, tg, ct, ocfg.steps)
    gm.forward_backward(*dev)
    loss = gm.loss()
    want = np.array([res["loss"], res["attn"], res["ctc"]])
    assert np.allclose(loss, want, rtol=1e-6, atol=0), (loss, want)
    for k, v in orc.debug.items():
        g = gm.debug_tensor(k, v.size)
        assert np.array_equal(g, v.ravel().astype(np.float32)), f"{k} differs"
    _compare(man, gm.get_grads(), orc.g, 1e-6, "gradient")
    gm.optimizer_step()
    _compare(man, gm.get_params(), orc.p, 1e-6, "updated parameter")
    assert lib.trba_tc_error_poll(1) == 0
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


@pytest.mark.parametrize("geom,B,fixed_len", [
    (dict(img_w=64, max_len=4), 48, 4),      # TRBA-small step: 32x64, batch 48, labels of length 4
    (dict(img_w=160, max_len=20), 48, None),  # 32x160, max_len 20, batch 48
    (dict(img_w=256, max_len=40), 48, None),  # 32x256, max_len 40, 48 lines per GPU (T = 32: CTC with L up to 41)
    (dict(img_w=160, max_len=20), 512, None),  # 32x160, batch 512: the benchmark's per-GPU batch
], ids=["32x64_L4_b48", "32x160_L20_b48", "32x256_L40_b48", "32x160_L20_b512"])
def test_benchmark_configurations_match_oracle(geom, B, fixed_len, lib, cuda):
    """One forward + backward + optimiser step at the benchmark's own
    configurations, bit for bit against the oracle (exact input gradient)."""
    ocfg, params, gm, man = _setup(geom, B, seed=2024, dgrad_mode=0)
    img, ti, tg, ct = so.make_batch(ocfg, B, seed=77, fixed_len=fixed_len)
    orc = so.OracleTrba(ocfg, params, _oracle_backend())
    res = orc.train_step(img, ti, tg, ct)
    gm.forward_backward(*_to_dev(img, ti, tg, ct, ocfg.steps))
    want = np.array([res["loss"], res["attn"], res["ctc"]])
    assert np.allclose(gm.loss(), want, rtol=1e-6, atol=0), (gm.loss(), want)
    for k in ("feat", "logits", "ctc_logits", "dfeat"):
        v = orc.debug[k]
        assert np.array_equal(gm.debug_tensor(k, v.size), v.ravel().astype(np.float32)), f"{k} differs"
    _compare(man, gm.get_grads(), orc.g, 1e-6, "gradient")
    gm.optimizer_step()
    _compare(man, gm.get_params(), orc.p, 1e-6, "updated parameter")
    assert lib.trba_tc_error_poll(1) == 0
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


def test_running_stats_follow_the_batch_statistics(lib, cuda):
    geom = dict(img_w=64, max_len=4)
    ocfg, params, gm, man = _setup(geom, 8, seed=5)
    img, ti, tg, ct = so.make_batch(ocfg, 8, seed=7)
    orc = so.OracleTrba(ocfg, params, _oracle_backend())
    orc.train_step(img, ti, tg, ct)
    gm.forward_backward(*_to_dev(img, ti, tg, ct, ocfg.steps))
    got = gm.running_stats()
    want = np.concatenate([np.concatenate([orc.run_mean[c.name], orc.run_var[c.name]]) for c in so.conv_specs(ocfg)])
    assert np.allclose(got, want, rtol=1e-6, atol=1e-7)


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


def test_loss_curve_200_steps_matches_oracle(lib, cuda):
    """Training loss within 1% of the reference's over 200 steps (the
    convergence bar of this port; TRBA-small 32x64, batch 8, a fresh
    synthetic batch every step)."""
    geom = dict(img_w=64, max_len=4)
    ocfg, params, gm, man = _setup(geom, 8, seed=21)
    orc = so.OracleTrba(ocfg, params, _oracle_backend())
    lo, lg = [], []
    for i in range(200):
        img, ti, tg, ct = so.make_batch(ocfg, 8, seed=1000 + i)
        lo.append(orc.train_step(img, ti, tg, ct)["loss"])
        gm.train_step(*_to_dev(img, ti, tg, ct, ocfg.steps))
        lg.append(float(gm.loss()[0]))
    lo, lg = np.array(lo), np.array(lg)
    rel = np.abs(lg - lo) / np.abs(lo)
    assert rel.max() < 0.01, f"max relative loss gap {rel.max():.3g} at step {int(rel.argmax())}"
    assert np.mean(lo[-20:]) < np.mean(lo[:20]), "the oracle's loss did not decrease"


def test_graph_replay_equals_eager_steps(lib, cuda):
    """trba_model_use_graphs: the step recorded once as a CUDA graph and
    replayed (inputs refreshed in place) gives bit-identical losses and
    parameters to eager steps, through both entry points."""
    import torch
    import trba_b200.model as tm
    geom = dict(img_w=64, max_len=4)
    ocfg, params, eager, man = _setup(geom, 8, seed=41)
    _, _, graph, _ = _setup(geom, 8, seed=41)
    graph.use_graphs(True)
    bufs = None
    for i in range(6):
        img, ti, tg, ct = so.make_batch(ocfg, 8, seed=300 + i)
        dev = _to_dev(img, ti, tg, ct, ocfg.steps)
        eager.train_step(*dev)
        if bufs is None:
            bufs = [d.clone() for d in dev]
        else:
            for b, d in zip(bufs, dev):
                b.copy_(d)
        graph.train_step(*bufs)
        assert np.array_equal(eager.loss(), graph.loss()), f"step {i}"
    assert np.array_equal(eager.get_params(), graph.get_params())
    assert lib.trba_model_step_count(graph.h) == 6
    for i in range(3):  # host-buffer entry point: one graph over the model's staging buffers
        img, ti, tg, ct = so.make_batch(ocfg, 8, seed=400 + i)
        host = (np.ascontiguousarray(img), *tm.pack_labels(ti, tg, ct, ocfg.steps))
        l1 = eager.train_step_host(*host)
        l2 = graph.train_step_host(*host)
        assert np.array_equal(l1, l2)
    assert np.array_equal(eager.get_params(), graph.get_params())
    torch.cuda.synchronize()
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


@pytest.mark.parametrize("version", [6, 5, 4])
def test_checkpoint_resume_equals_uninterrupted_training(version, lib, cuda, tmp_path):
    """TRBA_V6 written (and V5 / V4 derived from it as the reference lays them
    out) and read back into a fresh model: training continues exactly as the
    uninterrupted model (V4 carries no Adam moments, so only V6 / V5 resume
    bit-identically; V4 restores weights, BN statistics and the step)."""
    import struct
    import trba_b200.checkpoint as ck
    geom = dict(img_w=64, max_len=4)
    ocfg, params, a, man = _setup(geom, 8, seed=61)
    batches = [so.make_batch(ocfg, 8, seed=500 + i) for i in range(4)]
    for bt in batches[:2]:
        a.train_step(*_to_dev(*bt, ocfg.steps))
    path = tmp_path / "model.ckpt"
    ck.save(a, path, epoch_done=3, batch_in_epoch=17)
    if version < 6:  # rewrite into the older layouts
        full = ck.read(path)
        with open(path, "wb") as f:
            f.write(ck.MAGIC_V5 if version == 5 else ck.MAGIC_V4)
            f.write(struct.pack("<Q", full["epoch_done"]))
            if version == 5:
                f.write(struct.pack("<Q", full["batch_in_epoch"]))
            f.write(struct.pack("<Q", full["opt_t"]))
            f.write(struct.pack("<Q", len(full["params"])))
            for _, val, m, v in full["params"]:
                for arr in ((val, m, v) if version == 5 else (val,)):
                    f.write(struct.pack("<Q", arr.size) + arr.astype("<f4").tobytes())
            for rm, rv, cm, cv in full["convs"]:
                for arr in ((rm, rv, cm, cv) if version == 5 else (rm, rv)):
                    f.write(struct.pack("<Q", arr.size) + arr.astype("<f4").tobytes())
    _, _, b, _ = _setup(geom, 8, seed=999)  # different weights: everything must come from the file
    meta = ck.load(b, path)
    assert meta["version"] == version and meta["opt_t"] == 2 and meta["epoch_done"] == 3
    assert np.array_equal(a.get_params(), b.get_params())
    assert np.array_equal(a.running_stats(), b.running_stats())
    assert b.step_count() == 2
    for bt in batches[2:]:
        a.train_step(*_to_dev(*bt, ocfg.steps))
        b.train_step(*_to_dev(*bt, ocfg.steps))
    if version >= 5:
        assert np.array_equal(a.get_params(), b.get_params())
        assert np.array_equal(a.loss(), b.loss())
