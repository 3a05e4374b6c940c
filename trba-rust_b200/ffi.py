"""ctypes binding of libtrba_b200.so.

The argument and return types are read from the C headers in ``include/``
(the drop-in ABI of trba-rust's src/backend.rs plus this library's own
entry points), so the Python binding can never drift from the declarations a
Rust/C caller links against.  Loading fails loudly when the library has not
been built: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
LIB_PATH = HERE / "libtrba_b200.so"
HEADERS = sorted((REPO / "include").glob("*.h"))

_SCALARS = {
    "void": None,
    "int": C.c_int,
    "unsigned": C.c_uint,
    "size_t": C.c_size_t,
    "long long": C.c_longlong,
    "unsigned long long": C.c_ulonglong,
    "uint64_t": C.c_uint64,
    "int64_t": C.c_int64,
    "uint32_t": C.c_uint32,
    "int32_t": C.c_int32,
    "float": C.c_float,
    "double": C.c_double,
}

_DECL = re.compile(r"^\s*([A-Za-z_][\w \*]*?[\s\*])([A-Za-z_]\w*)\s*\(([^;]*?)\)\s*;", re.M | re.S)


def _ctype(t: str):
    t = " ".join(t.replace("const", " ").split())
    if t.endswith("*"):
        base = t.rstrip("*").strip()
        return C.c_char_p if base == "char" and t.count("*") == 1 else C.c_void_p
    if t not in _SCALARS:
        raise ValueError(f"unsupported C type in header: {t!r}")
    return _SCALARS[t]


def parse_header(text: str) -> dict[str, tuple]:
    """name -> (restype, [argtypes]) for every function declared in `text`."""
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    text = re.sub(r"^\s*#.*$", " ", text, flags=re.M)
    out = {}
    for m in _DECL.finditer(text):
        ret, name, args = m.group(1), m.group(2), m.group(3)
        if name in ("if", "while", "for", "return"):
            continue
        argtypes = []
        args = " ".join(args.split())
        if args and args != "void":
            for a in args.split(","):
                a = a.strip()
                if "(*" in a:  # function pointer (one parameter each in these headers): passed as an address
                    argtypes.append(C.c_void_p)
                    continue
                am = re.match(r"^(.*?[\s\*])([A-Za-z_]\w*)$", a)
                argtypes.append(_ctype(am.group(1) if am else a))
        out[name] = (_ctype(ret.strip()), argtypes)
    return out


def declared_functions() -> dict[str, tuple]:
    decls = {}
    for h in HEADERS:
        decls.update(parse_header(h.read_text()))
    return decls


_LIB = None


def lib() -> C.CDLL:
    """The loaded library with every header-declared symbol typed."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it first (python __graft_entry__.py build, "
            "or trba-rust_b200/build.py). There is no CPU fallback.")
    L = C.CDLL(str(LIB_PATH))
    for name, (res, args) in declared_functions().items():
        f = getattr(L, name)  # AttributeError here means the .so lacks a declared symbol
        f.restype = res
        f.argtypes = args
    _LIB = L
    return L
