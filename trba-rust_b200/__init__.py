"""trba_b200 — B200-native (sm_100a) INT8-QAT hot path of trba-rust.

The product is ``libtrba_b200.so``: the reference's backend C ABI
(src/backend.rs) and a fused, device-resident QAT training step, written as
CUDA kernels for sm_100a.  This Python package is a thin ctypes binding used
by the tests, the benchmark and anyone who drives the library from Python.
"""
from .ffi import lib, declared_functions, LIB_PATH  # noqa: F401

__all__ = ["lib", "declared_functions", "LIB_PATH"]
