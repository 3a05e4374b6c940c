"""The model's conv forward with the implicit GEMM (conv_fwd_mode = 1, the
default) against the im2col matrix + GEMM (conv_fwd_mode = 0) on identical
weights and inputs.

In training the implicit GEMM's forward writes no im2col matrix; the weight
gradient's operand (the matrix for the reference-compatible weight gradient,
wgrad_mode = 0, its transpose for wgrad_mode = 1) is built on the
weight-gradient stream while the sequence head runs.  The s32 accumulators
and the operands are equal either way, so losses,
every parameter gradient, parameters after an optimiser step, and the greedy
tokens must be bit-identical between the two modes."""
import sys

import numpy as np
import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))
import step_oracle as so  # noqa: E402

pytestmark = pytest.mark.gpu


def _models(geom, B, seed, **kw):
    import trba_b200.model as tm
    ocfg = so.Config(**geom)
    params = so.init_params(ocfg, seed)
    flat = np.concatenate([params[n].ravel() for n, _, _ in so.manifest(ocfg)]).astype(np.float32)
    ms = []
    for mode in (0, 1):
        m = tm.QatModel(tm.Config(**geom, batch=B, conv_fwd_mode=mode, **kw))
        m.set_params(flat)
        ms.append(m)
    return ocfg, ms


@pytest.mark.parametrize("wgrad_mode", [0, 1])
@pytest.mark.parametrize("geom,B", [(dict(img_w=64, max_len=4), 8), (dict(img_w=160, max_len=20), 4)],
                         ids=["32x64_b8", "32x160_b4"])
def test_training_steps_agree_between_forward_modes(geom, B, wgrad_mode, lib, cuda):
    import torch
    import trba_b200.model as tm
    ocfg, (a, b) = _models(geom, B, seed=19, wgrad_mode=wgrad_mode, dgrad_mode=1)
    for step in range(2):
        img, ti, tg, ct = so.make_batch(ocfg, B, seed=300 + step)
        ti32, tg32, ctc, lens = tm.pack_labels(ti, tg, ct, ocfg.steps)
        dev = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (img, ti32, tg32, ctc, lens)]
        a.forward_backward(*dev)
        b.forward_backward(*dev)
        assert np.array_equal(a.loss(), b.loss())
        assert np.array_equal(a.get_grads(), b.get_grads())
        a.optimizer_step()
        b.optimizer_step()
        assert np.array_equal(a.get_params(), b.get_params())
        assert np.array_equal(a.running_stats(), b.running_stats())
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


@pytest.mark.parametrize("per_channel", [0, 1])
def test_inference_agrees_between_forward_modes(per_channel, lib, cuda):
    geom = dict(img_w=160, max_len=20)
    ocfg, (a, b) = _models(geom, 16, seed=23, wq_per_channel=per_channel, inference_only=1)
    rng = np.random.default_rng(5)
    rs = np.concatenate([np.stack([rng.standard_normal(c) * 0.1, 0.5 + rng.random(c)]).ravel()
                         for c in a.conv_channels()]).astype(np.float32)
    a.set_running_stats(rs)
    b.set_running_stats(rs)
    img, _, _, _ = so.make_batch(ocfg, 16, seed=77)
    assert a.infer_host(img) == b.infer_host(img)
    T = geom["img_w"] // 8  # encoder steps: the last conv's output width
    feat = [m.debug_tensor("feat", 16 * T * ocfg.fd) for m in (a, b)]
    assert np.array_equal(feat[0], feat[1])
    for name, n in (("layer2.1.conv2.x", 16 * 64 * 8 * 40), ("layer4.2.conv2.x", 16 * 128 * 4 * 20)):
        assert np.array_equal(a.debug_tensor(name, n), b.debug_tensor(name, n)), name
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()
