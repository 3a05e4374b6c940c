"""The CTA-pair int8 GEMM (tcgen05 cta_group::2, 256 x 256 tiles over two
SMs) that serves large unsplit problems: s32 results bit-identical to exact
f64 products and to the single-CTA kernel on the same operands, and the
fused requant / dequant epilogues identical between the two paths."""
import ctypes as C

import numpy as np
import pytest

SHAPES = [(24613, 512, 600), (98304, 256, 1152), (37000, 768, 136)]


def _inputs(torch, m, n, k, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    kp = (k + 15) // 16 * 16
    a = torch.zeros((m, kp), dtype=torch.int8)
    b = torch.zeros((n, kp), dtype=torch.int8)
    a[:, :k] = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b[:, :k] = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    return a.cuda(), b.cuda()


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_pair_gemm_s32_exact(shape, lib, cuda):
    import torch
    m, n, k = shape
    a, b = _inputs(torch, m, n, k, seed=m + n + k)
    want = (a[:, :k].to(torch.float64) @ b[:, :k].to(torch.float64).t()).to(torch.int32)
    got = torch.full((m, n), -7, dtype=torch.int32, device=cuda)
    assert lib.trba_gemm_pair_enable(1) in (0, 1)
    lib.launch_gemm_int8(_p(a), _p(b), _p(got), m, n, k, None)
    single = torch.full((m, n), -7, dtype=torch.int32, device=cuda)
    lib.trba_gemm_pair_enable(0)
    lib.launch_gemm_int8(_p(a), _p(b), _p(single), m, n, k, None)
    lib.trba_gemm_pair_enable(1)
    torch.cuda.synchronize()
    assert lib.trba_tc_error_poll(1) == 0
    assert torch.equal(got, want)
    assert torch.equal(single, want)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES[:2], ids=lambda s: "x".join(map(str, s)))
def test_pair_gemm_fused_epilogues_match_single_cta(shape, lib, cuda):
    import torch
    m, n, k = shape
    a, b = _inputs(torch, m, n, k, seed=3 * m + n)
    g = np.random.default_rng(n)
    bias = torch.from_numpy(g.uniform(-1, 1, n).astype(np.float32)).cuda()
    w_scale = torch.from_numpy(np.exp(g.uniform(np.log(1e-4), np.log(1e-1), n)).astype(np.float32)).cuda()
    outs = {}
    for pair in (1, 0):
        lib.trba_gemm_pair_enable(pair)
        rq = torch.full((m, n), 99, dtype=torch.int8, device=cuda)
        lib.trba_gemm_int8_requant(_p(a), _p(b), _p(bias), _p(rq), m, n, k, 127.0 * 64.0, 50.0, None)
        dq = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
        lib.trba_gemm_int8_dequant_f32(_p(a), _p(b), _p(w_scale), float(np.float32(1.0 / 127.0)), _p(bias), 1,
                                       _p(dq), m, n, k, None)
        outs[pair] = (rq, dq)
    lib.trba_gemm_pair_enable(1)
    torch.cuda.synchronize()
    assert lib.trba_tc_error_poll(1) == 0
    assert torch.equal(outs[1][0], outs[0][0])
    assert torch.equal(outs[1][1], outs[0][1])
