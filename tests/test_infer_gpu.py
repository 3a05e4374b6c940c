"""Inference (run_inference / greedy_decode of the reference): the device
path (trba_model_infer / trba_model_infer_host) against the oracle's eval
forward and greedy decoding on the same weights, running statistics and
images.  The eval forward reuses the training kernels with the BN running
statistics, so logits and argmax tokens are bit-identical."""
import sys

import numpy as np
import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))
import step_oracle as so  # noqa: E402

pytestmark = pytest.mark.gpu


def _pair(geom, B, seed, train_steps):
    import torch
    import trba_b200.model as tm
    ocfg = so.Config(**geom)
    params = so.init_params(ocfg, seed)
    gm = tm.QatModel(tm.Config(**geom, batch=B))
    names = [n for n, _, _ in so.manifest(ocfg)]
    gm.set_params(np.concatenate([params[n].ravel() for n in names]).astype(np.float32))
    orc = so.OracleTrba(ocfg, params, so.CpuBackend(REPO / "oracle" / "liboracle.so"))
    for i in range(train_steps):  # a few identical training steps: non-trivial running statistics
        img, ti, tg, ct = so.make_batch(ocfg, B, seed=900 + i)
        orc.train_step(img, ti, tg, ct)
        ti32, tg32, ctc, lens = tm.pack_labels(ti, tg, ct, ocfg.steps)
        dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (img, ti32, tg32, ctc, lens)]
        gm.train_step(*dev)
    return ocfg, orc, gm


@pytest.mark.parametrize("geom,B,steps", [(dict(img_w=64, max_len=4), 8, 3), (dict(img_w=160, max_len=20), 4, 2)],
                         ids=["32x64_b8", "32x160_b4"])
def test_greedy_decoding_matches_oracle(geom, B, steps, lib, cuda):
    import torch
    ocfg, orc, gm = _pair(geom, B, seed=77, train_steps=steps)
    img, _, _, _ = so.make_batch(ocfg, B, seed=1234)
    want_lists, want_steps = orc.infer(img)
    got_steps = gm.infer(torch.from_numpy(np.ascontiguousarray(img)).cuda())
    ran = want_steps[:, 0] >= 0  # the oracle stops at the first all-eos step
    assert np.array_equal(got_steps[ran], want_steps[ran])
    assert gm.infer_host(img) == want_lists
    other, _, _, _ = so.make_batch(ocfg, B, seed=4321)
    gm.infer_host(other)  # an unrelated call in between leaves no trace
    assert gm.infer_host(img) == want_lists
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


def test_inference_leaves_training_state_alone(lib, cuda):
    """Inference reads the running statistics and parameters; it changes
    neither, and a training step after it equals one without it."""
    import torch
    import trba_b200.model as tm
    geom = dict(img_w=64, max_len=4)
    ocfg, _, a = _pair(geom, 8, seed=5, train_steps=1)
    _, _, b = _pair(geom, 8, seed=5, train_steps=1)
    img, ti, tg, ct = so.make_batch(ocfg, 8, seed=31)
    rs, p = a.running_stats(), a.get_params()
    a.infer_host(img)
    assert np.array_equal(a.running_stats(), rs) and np.array_equal(a.get_params(), p)
    ti32, tg32, ctc, lens = tm.pack_labels(ti, tg, ct, ocfg.steps)
    dev = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (img, ti32, tg32, ctc, lens)]
    a.train_step(*dev)
    b.train_step(*dev)
    assert np.array_equal(a.get_params(), b.get_params())
