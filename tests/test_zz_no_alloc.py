"""The GEMM entry point that allocates nothing (trba_sgemm_exact_noalloc).

It exists for callers that may not allocate device memory themselves —
plugins whose host framework owns every device allocation, or loops in which
a cudaMalloc / cudaFree would synchronise the device.  Its split-K scratch
is a static device array inside the library instead of a buffer it would
allocate.

Checked through the C ABI against the existing fp32 GEMM entry point
(launch_gemm_fp32, same contract: A [M,K] @ B [K,N] -> C [M,N]) within the
fp32-GEMM tolerance the ABI tests use (1e-5 relative), and against an f64
reference (it accumulates in f64), on two calls in a row: the second call
reuses the scratch the first one left behind.  This file is collected last
so that a run stopping at its first failure has run everything else first.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("shapes", [[(300, 200, 5000), (64, 130, 20000)], [(129, 65, 777), (129, 65, 777)]],
                         ids=["two_shapes", "same_shape_twice"])
def test_noalloc_gemm_matches_existing_entry_point(shapes, lib, cuda):
    import torch
    g = torch.Generator(device="cpu").manual_seed(7)
    for call, (m, n, k) in enumerate(shapes):
        a = torch.randn(m, k, generator=g).float().cuda()
        b = torch.randn(k, n, generator=g).float().cuda()
        c_ref = torch.full((m, n), 9.0, device="cuda")
        c_new = torch.full((m, n), -9.0, device="cuda")
        lib.launch_gemm_fp32(_p(a), _p(b), _p(c_ref), m, n, k, None)
        rc = lib.trba_sgemm_exact_noalloc(_p(a), _p(b), _p(c_new), m, n, k, None)
        torch.cuda.synchronize()
        assert rc == 0, lib.trba_last_error_string()
        want = c_ref.cpu().numpy().astype(np.float64)
        got = c_new.cpu().numpy().astype(np.float64)
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), f"call {call}"
        exact = a.double().cpu().numpy() @ b.double().cpu().numpy()
        assert np.abs(got - exact).max() <= 1e-6 * max(1.0, np.abs(exact).max()), f"call {call} vs f64"
    assert lib.trba_last_error() == 0, lib.trba_last_error_string()


def test_noalloc_gemm_rejects_sizes_beyond_its_scratch(lib, cuda):
    lib.trba_clear_error()
    rc = lib.trba_sgemm_exact_noalloc(None, None, None, 1024, 1024, 8, None)
    assert rc == -1
    assert b"131072" in lib.trba_last_error_string()
    lib.trba_clear_error()
