"""Shared fixtures: the product library (libtrba_b200.so, via the trba_b200
package), the CPU oracle (oracle/liboracle.so, test infrastructure only) and
the reference's own CPU backend (oracle/_ref/, when it was built here)."""
from __future__ import annotations

import ctypes as C
import importlib.util
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

try:  # load PyTorch (and its CUDA / NCCL libraries) before libtrba_b200
    import torch  # noqa: F401
except Exception:  # pragma: no cover
    torch = None

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: multi-second CPU oracle runs")


def load_package():
    name = "trba_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = REPO / "trba-rust_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()


def _typed_cpu_backend(path: Path) -> C.CDLL:
    """A CPU backend with the reference's ABI (oracle or reference build),
    typed from include/trba_backend.h."""
    from trba_b200.ffi import parse_header
    L = C.CDLL(str(path))
    decls = parse_header((REPO / "include" / "trba_backend.h").read_text())
    for name, (res, args) in decls.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
    return L


@pytest.fixture(scope="session")
def oracle():
    so = REPO / "oracle" / "liboracle.so"
    if not so.exists():
        subprocess.run(["make", "-C", str(REPO / "oracle"), "oracle"], check=True,
                       capture_output=True)
    return _typed_cpu_backend(so)


@pytest.fixture(scope="session")
def ref_cpu():
    so = REPO / "oracle" / "_ref" / "libtrba_ref_omp.so"
    if not so.exists():
        pytest.skip("reference CPU backend not built (oracle/_ref absent)")
    return _typed_cpu_backend(so)


@pytest.fixture(scope="session")
def lib():
    import trba_b200
    L = trba_b200.lib()
    L.trba_set_abort_on_error(0)
    return L


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "ref_kat.npz"))
