"""MoPE length-bucket serving (trba_b200.mope): routing, placement and the
greedy output rule on CPU; on the GPU, an expert's served output equals the
model's own host-buffer inference and the oracle's greedy decoding."""
import sys

import numpy as np
import pytest

from conftest import REPO

sys.path.insert(0, str(REPO / "oracle"))
import step_oracle as so  # noqa: E402


def test_route_by_length_bucket():
    import trba_b200.mope as mp
    ex = mp.default_experts()
    assert len(ex) == 9
    r = mp.route([1, 4, 5, 9, 11, 12, 13, 32, 99], ex)
    assert r == [0, 0, 1, 5, 7, 7, 8, 8, 8]


def test_place_balances_expected_work():
    import trba_b200.mope as mp
    ex = mp.default_experts()
    lens = mp.synthetic_lengths(65536, seed=3)
    counts = np.bincount(mp.route(lens, ex), minlength=len(ex)).tolist()
    assert sum(counts) == 65536
    for world in (1, 2, 4, 8):
        plan = mp.place(ex, counts, world)
        assert set(plan) <= set(range(world))
        load = [0.0] * world
        for i, r in enumerate(plan):
            load[r] += mp.expected_work(ex[i], counts[i])
        biggest = max(mp.expected_work(e, c) for e, c in zip(ex, counts))
        # greedy LPT: no rank exceeds the mean load by more than one expert
        assert max(load) <= sum(load) / world + biggest + 1e-9
        if world == 1:
            assert plan == [0] * 9


def test_synthetic_lengths_follow_the_documented_quantiles():
    import trba_b200.mope as mp
    v = np.array(mp.synthetic_lengths(200000, seed=1))
    assert abs(np.median(v) - 5) <= 1 and abs(np.quantile(v, 0.9) - 11) <= 1.5 and v.max() <= 32 and v.min() >= 1


def test_decode_rule_matches_the_reference_loop():
    """src/attn.rs:423-443 restated as a loop over steps with early exit."""
    import trba_b200.mope as mp
    rng = np.random.default_rng(0)
    eos = 2
    for _ in range(200):
        steps, n = rng.integers(1, 8), rng.integers(1, 5)
        st = rng.integers(0, 5, size=(steps, n)).astype(np.int32)
        want = [[] for _ in range(n)]
        for s in range(steps):
            all_eos = True
            for b in range(n):
                if st[s, b] == eos:
                    continue
                all_eos = False
                want[b].append(int(st[s, b]))
            if all_eos:
                break
        assert mp.decode_rule(st, eos) == want


@pytest.mark.gpu
def test_expert_serving_equals_model_inference_and_oracle(lib, cuda):
    import torch
    import trba_b200.mope as mp
    e = mp.Expert("bucket_04_04", 4, 4, 64, 4)
    run = mp.ExpertRunner(e, batch=8, seed=11)  # inference-only, per-channel int8 weights
    ocfg = so.Config(img_w=64, max_len=4, wq_per_channel=True)
    imgs = [so.make_batch(ocfg, 8, seed=70 + i)[0] for i in range(2)]
    dev = torch.from_numpy(np.ascontiguousarray(np.concatenate(imgs))).cuda()
    served = run.decode(dev)
    host = run.model.infer_host(imgs[0]) + run.model.infer_host(imgs[1])
    assert served == host
    from trba_b200.data import init_params
    params = init_params(run.model.manifest(), run.cfg, 11)
    names = [n for n, _, _ in so.manifest(ocfg)]
    off = 0
    pd = {}
    for n, shape, _ in so.manifest(ocfg):
        k = int(np.prod(shape))
        pd[n] = params[off:off + k].reshape(shape)
        off += k
    orc = so.OracleTrba(ocfg, pd, so.CpuBackend(REPO / "oracle" / "liboracle.so"))
    want = orc.infer(imgs[0])[0] + orc.infer(imgs[1])[0]
    assert served == want
    run.close()


@pytest.mark.gpu
def test_inference_only_expert_refuses_training_and_is_smaller(lib, cuda):
    """An inference-only expert holds the forward path only: no gradients,
    optimiser state or backward traces, and every training entry point
    returns -3 instead of touching them."""
    import trba_b200.model as tm
    from trba_b200.data import init_params
    cfg = tm.Config(img_w=256, max_len=40, batch=64, wq_per_channel=1, inference_only=1)
    inf = tm.QatModel(cfg)
    tr = tm.QatModel(tm.Config(img_w=256, max_len=40, batch=64, wq_per_channel=1))
    bi, bt = int(lib.trba_model_device_bytes(inf.h)), int(lib.trba_model_device_bytes(tr.h))
    assert bi < 0.75 * bt, (bi, bt)
    inf.set_params(init_params(inf.manifest(), cfg, 3))
    lib.trba_set_abort_on_error(0)
    assert lib.trba_model_optimizer_step(inf.h, None) == -3
    g = np.empty(inf.n_params, np.float32)
    assert lib.trba_model_get_grads(inf.h, g.ctypes.data, g.size) == -3
    lib.trba_clear_error()
    import torch
    img = torch.zeros((4, 3, 32, 256), dtype=torch.int8, device="cuda")
    tok = inf.infer(img)
    assert tok.shape == (41, 4)
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()
    inf.close()
    tr.close()
