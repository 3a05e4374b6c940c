"""The drop-in boundary: libtrba_b200.so exports every function the C
headers declare, and the headers declare every symbol of the reference's
backend ABI (the 76 exports of its cuda/kernels.cu / cpu_backend.cpp, listed
in tests/golden/ref_symbols.txt).  CPU only: nothing here launches a kernel."""
import ctypes as C
import subprocess

import pytest

from conftest import GOLDEN, REPO


def test_library_loads_and_exports_every_declared_symbol():
    import trba_b200
    decls = trba_b200.declared_functions()
    L = trba_b200.lib()
    missing = [n for n in decls if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert L.trba_backend_name() == b"b200-sm100a"


def test_headers_cover_the_reference_abi():
    import trba_b200
    ref = set((GOLDEN / "ref_symbols.txt").read_text().split())
    assert len(ref) == 76
    decls = set(trba_b200.declared_functions())
    assert ref - decls == set()


def test_exports_match_nm():
    so = REPO / "trba-rust_b200" / "libtrba_b200.so"
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
    exported = {l.split()[2] for l in out.splitlines() if len(l.split()) == 3 and l.split()[1] == "T"}
    ref = set((GOLDEN / "ref_symbols.txt").read_text().split())
    assert ref <= exported


def test_sticky_error_mode_reports_bad_shapes(lib):
    # A shape the reference rejects (odd H for the 2x2 pool) must not launch:
    # with abort disabled it lands in the error word instead.
    lib.trba_clear_error()
    lib.launch_maxpool2x2_forward_i8(None, None, 1, 1, 3, 4, None)
    assert lib.trba_last_error() != 0
    assert b"maxpool" in lib.trba_last_error_string()
    lib.trba_clear_error()
    assert lib.trba_last_error() == 0


def test_non_positive_sizes_return_silently(lib):
    lib.trba_clear_error()
    lib.launch_gemm_int8(None, None, None, 0, 5, 5, None)
    lib.launch_quant_f32_i8(None, 0, 1.0, None, None)
    assert lib.trba_last_error() == 0
