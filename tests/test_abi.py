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


def test_static_archive_links_like_the_reference_backend(tmp_path):
    """libtrba_cuda.a (the archive name the reference's build.rs links) holds
    every declared function, and a C program calling the reference ABI links
    against it with the reference's own link line (static cudart, stdc++, m,
    dl, rt, pthread).  Linking only: nothing runs."""
    import trba_b200
    ar = REPO / "trba-rust_b200" / "libtrba_cuda.a"
    assert ar.exists(), "static archive not built"
    out = subprocess.run(["nm", "-g", "--defined-only", str(ar)], capture_output=True, text=True).stdout
    defined = {l.split()[2] for l in out.splitlines() if len(l.split()) == 3 and l.split()[1] == "T"}
    missing = [n for n in trba_b200.declared_functions() if n not in defined]
    assert not missing, missing
    src = tmp_path / "main.c"
    src.write_text('#include "trba_backend.h"\n#include "trba_qat.h"\n'
                   "int main(void) { trba_model_config c; trba_model_default_config(&c);\n"
                   "  launch_gemm_int8(0, 0, 0, 0, 0, 0, 0); return c.fd == 128 ? 0 : 1; }\n")
    cuda_lib = "/usr/local/cuda/lib64"
    r = subprocess.run(["g++", "-o", str(tmp_path / "a.out"), "-x", "c", str(src), "-x", "none",
                        f"-I{REPO / 'include'}", str(ar), f"-L{cuda_lib}", "-lcudart_static", "-lstdc++", "-lm",
                        "-ldl", "-lrt", "-lpthread"], capture_output=True, text=True)
    if r.returncode != 0 and "cannot find -lcudart_static" in r.stderr:
        pytest.skip("CUDA toolkit's static runtime not installed here")
    assert r.returncode == 0, r.stderr[-2000:]


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
