"""Parity of libtrba_b200.so's drop-in ABI on the GPU.

1. The reference unit tests' known answers (tests/golden/ref_kat.npz).
2. Every seeded case of tests/abi_cases.py against the CPU oracle (itself
   pinned to the reference's CPU backend by tests/test_oracle_golden.py).
3. The tcgen05 int8 GEMM over the reference's GEMM sweep shapes
   (M in {6144, 24576, 98304}, N in {64..512}, K in {64..2304}): s32 bit-exact
   against cuBLAS int8 (torch._int_mm) on the full result and against the
   CPU oracle on a sample of rows, plus odd shapes and the CUDA-core fallback.
"""
import ctypes as C

import numpy as np
import pytest

import abi_cases
from kat_runner import CudaBackend, HostBackend, compare, run_kat

pytestmark = pytest.mark.gpu


def test_known_answers_on_gpu(lib, cuda, golden):
    got = run_kat(CudaBackend(lib))
    bad = compare(got, golden)
    assert not bad, "\n".join(bad)
    assert lib.trba_tc_error_poll(1) == 0
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


@pytest.mark.parametrize("case", list(abi_cases.cases()), ids=lambda c: c[0])
def test_abi_matches_oracle(case, lib, cuda, oracle):
    cid, fn, args = case
    want = abi_cases.run_case(HostBackend(oracle), fn, args)
    got = abi_cases.run_case(CudaBackend(lib), fn, args)
    msgs = abi_cases.compare_outputs(got, want)
    assert not msgs, f"{cid}: " + "; ".join(msgs)
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


SWEEP = [(m, n, k) for m in (6144, 24576, 98304) for n in (64, 128, 256, 512) for k in (64, 576, 1152, 2304)]


def _gemm_inputs(torch, m, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = (k + 15) & ~15
    a = torch.randint(-127, 128, (m, kp), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (n, kp), dtype=torch.int8, device="cuda", generator=g)
    a[:, k:] = 0
    b[:, k:] = 0
    return a, b


@pytest.mark.parametrize("shape", SWEEP, ids=lambda s: "x".join(map(str, s)))
def test_gemm_sweep_bit_exact(shape, lib, cuda, oracle):
    import torch
    m, n, k = shape
    a, b = _gemm_inputs(torch, m, n, k, seed=m * 7 + n * 3 + k)
    c = torch.full((m, n), -1, dtype=torch.int32, device="cuda")
    lib.launch_gemm_int8(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(c.data_ptr()), m, n, k, None)
    want = torch._int_mm(a[:, :k].contiguous(), b[:, :k].t().contiguous())
    torch.cuda.synchronize()
    assert lib.trba_tc_error_poll(1) == 0
    assert torch.equal(c, want), f"{(c != want).sum().item()} mismatches"
    # CPU oracle on 48 sampled rows (the oracle's own padded-operand contract)
    rows = torch.randperm(m, device="cpu")[:48].sort().values
    a_s = a[rows.cuda()].cpu().numpy()
    b_h = b.cpu().numpy()
    c_s = np.zeros((48, n), dtype=np.int32)
    oracle.launch_gemm_int8(C.c_void_p(a_s.ctypes.data), C.c_void_p(b_h.ctypes.data),
                            C.c_void_p(c_s.ctypes.data), 48, n, k, None)
    assert np.array_equal(c[rows.cuda()].cpu().numpy(), c_s)


@pytest.mark.parametrize("shape", [(1, 1, 1), (17, 5, 3), (128, 32, 128), (129, 33, 129), (1000, 260, 300),
                                   (245760 // 16, 32, 144), (3840, 128, 1152), (2016, 128, 512), (7, 512, 2304)],
                         ids=lambda s: "x".join(map(str, s)))
def test_gemm_tails_and_conv_shapes(shape, lib, cuda):
    import torch
    m, n, k = shape
    a, b = _gemm_inputs(torch, m, n, k, seed=11 + m + n + k)
    c = torch.full((m, n), -1, dtype=torch.int32, device="cuda")
    lib.launch_gemm_int8(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(c.data_ptr()), m, n, k, None)
    want = (a[:, :k].to(torch.float64) @ b[:, :k].to(torch.float64).t()).to(torch.int32)
    torch.cuda.synchronize()
    assert torch.equal(c, want)
    # the CUDA-core fallback (used for operands a tensor map cannot describe)
    c2 = torch.full((m, n), -1, dtype=torch.int32, device="cuda")
    lib.trba_gemm_int8_simt(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(c2.data_ptr()), m, n, k,
                            None)
    torch.cuda.synchronize()
    assert torch.equal(c2, want)
    assert lib.trba_tc_error_poll(1) == 0


def test_gemm_unaligned_operand_takes_the_fallback(lib, cuda):
    import torch
    m, n, k = 70, 40, 48
    buf = torch.zeros(m * 48 + 16, dtype=torch.int8, device="cuda")
    a = buf[1:1 + m * 48].view(m, 48)  # base address 1 byte past a 16-byte boundary
    a.copy_(torch.randint(-127, 128, (m, 48), dtype=torch.int8, device="cuda"))
    b = torch.randint(-127, 128, (n, 48), dtype=torch.int8, device="cuda")
    c = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    lib.launch_gemm_int8(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(c.data_ptr()), m, n, k, None)
    want = (a.to(torch.float64) @ b.to(torch.float64).t()).to(torch.int32)
    torch.cuda.synchronize()
    assert torch.equal(c, want)


@pytest.mark.parametrize("shape", [(1, 1, 1), (17, 5, 3), (129, 33, 129), (1000, 260, 300), (6144, 512, 2304),
                                   (3840, 128, 1152), (200, 48, 64)],
                         ids=lambda s: "x".join(map(str, s)))
def test_fused_requant_epilogue_equals_gemm_then_conv_epilogue(shape, lib, cuda, oracle):
    """trba_gemm_int8_requant = launch_gemm_int8 + launch_conv_epilogue
    (cuda/kernels.cu:434-466) fused: int8 outputs bit-identical to the
    two-launch composition here and to the oracle's composition."""
    import torch
    m, n, k = shape
    a, b = _gemm_inputs(torch, m, n, k, seed=5 + m + n + k)
    g = torch.Generator(device="cpu").manual_seed(m + n)
    bias = (torch.rand(n, generator=g) * 2 - 1).float().cuda()
    div, mul = 127.0 * 64.0, 50.0
    fused = torch.full((m, n), 99, dtype=torch.int8, device="cuda")
    lib.trba_gemm_int8_requant(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(bias.data_ptr()),
                               C.c_void_p(fused.data_ptr()), m, n, k, div, mul, None)
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    lib.launch_gemm_int8(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(acc.data_ptr()), m, n, k,
                         None)
    two = torch.full((m, n), 99, dtype=torch.int8, device="cuda")
    lib.launch_conv_epilogue(C.c_void_p(acc.data_ptr()), C.c_void_p(bias.data_ptr()), C.c_void_p(two.data_ptr()), n,
                             div, mul, m, n, 1, 1, None)
    torch.cuda.synchronize()
    assert lib.trba_tc_error_poll(1) == 0
    assert torch.equal(fused, two)
    acc_h, bias_h = acc.cpu().numpy(), bias.cpu().numpy()
    want = np.zeros((m, n), np.int8)
    oracle.launch_conv_epilogue(C.c_void_p(acc_h.ctypes.data), C.c_void_p(bias_h.ctypes.data),
                                C.c_void_p(want.ctypes.data), n, div, mul, m, n, 1, 1, None)
    assert np.array_equal(fused.cpu().numpy(), want)


@pytest.mark.parametrize("shape", [(1, 1, 1), (129, 33, 129), (1000, 260, 300), (6144, 512, 2304)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("bias,relu", [(False, 0), (True, 1)], ids=["plain", "bias_relu"])
def test_fused_dequant_epilogue(shape, bias, relu, lib, cuda):
    """out = act((float)acc * (a_scale * w_scale[n]) + bias[n]), every
    operation an IEEE f32 multiply / add: bit-identical to numpy float32."""
    import torch
    m, n, k = shape
    a, b = _gemm_inputs(torch, m, n, k, seed=9 + m + n + k)
    g = np.random.default_rng(m * 3 + n)
    w_scale = np.exp(g.uniform(np.log(1e-4), np.log(1e-1), n)).astype(np.float32)
    bvec = g.uniform(-1, 1, n).astype(np.float32)
    a_scale = np.float32(1.0 / 127.0)
    ws_d = torch.from_numpy(w_scale).cuda()
    b_d = torch.from_numpy(bvec).cuda()
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    lib.trba_gemm_int8_dequant_f32(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(ws_d.data_ptr()),
                                   float(a_scale), C.c_void_p(b_d.data_ptr()) if bias else None, relu,
                                   C.c_void_p(out.data_ptr()), m, n, k, None)
    acc = (a[:, :k].to(torch.float64) @ b[:, :k].to(torch.float64).t()).to(torch.int32).cpu().numpy()
    torch.cuda.synchronize()
    assert lib.trba_tc_error_poll(1) == 0
    want = acc.astype(np.float32) * (a_scale * w_scale)[None, :]
    if bias:
        want = (want + bvec[None, :]).astype(np.float32)
    if relu:
        want = np.maximum(want, np.float32(0))
    assert np.array_equal(out.cpu().numpy(), want.astype(np.float32))
