"""Build recipe of libtrba_b200.so (sm_100a only).

Compiles every ``csrc/*.cu`` with nvcc for ``compute_100a``/``sm_100a`` into
``_build/`` and links the shared library in-tree next to this file, so it
travels with the source tree; the same objects also go into the static
archive ``libtrba_cuda.a`` (the archive name the reference's build.rs links).  Rebuilds only what changed (object newer than
its source and every header).  No PyTorch extension machinery: the library is
a plain C ABI and is loaded with ctypes.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libtrba_b200.so"
# The same objects as a static archive under the name the reference's
# build.rs links (cargo:rustc-link-lib=static=trba_cuda).
ARCHIVE = HERE / "libtrba_cuda.a"
REPO = HERE.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills", f"-I{REPO / 'include'}", f"-I{CSRC}",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: libtrba_b200 needs the CUDA toolkit to build")


def _nccl_dirs() -> tuple[list[str], list[str]]:
    """NCCL header location (system copy, else the wheel's).  The library is
    not linked against NCCL: it is dlopen'ed at run time."""
    inc, lib = [], ["-ldl"]
    if Path("/usr/include/nccl.h").exists():
        return inc, lib
    try:
        import nvidia.nccl as nn  # type: ignore
        root = Path(list(nn.__path__)[0])
        inc = [f"-I{root / 'include'}"]
    except Exception:
        pass
    return inc, lib


def build(verbose: bool = False, jobs: int = 8) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))
    newest_hdr = max((h.stat().st_mtime for h in headers), default=0.0)
    nccl_inc, nccl_lib = _nccl_dirs()

    def obj_of(src: Path) -> Path:
        return BUILD / (src.stem + ".o")

    def compile_one(src: Path) -> Path:
        obj = obj_of(src)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_hdr):
            return obj
        cmd = [nvcc, *NVCC_FLAGS, *nccl_inc, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, srcs))

    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", *[str(o) for o in objs], "-o", str(tmp),
               *nccl_lib]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if not ARCHIVE.exists() or ARCHIVE.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = ARCHIVE.with_suffix(".a.tmp")
        if tmp.exists():
            tmp.unlink()
        r = subprocess.run(["ar", "rcs", str(tmp), *[str(o) for o in objs]], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"ar failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, ARCHIVE)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
