"""Build libfhe_b200.so in-tree for sm_100a with nvcc.

``python -m fhe_mamba_b200.build`` (or ``build()``) compiles every
``csrc/*.cu`` to an object under ``_build/`` (skipping up-to-date objects) and
links ``fhe_mamba_b200/libfhe_b200.so``.  The library is kept in the source
tree so that it travels with the repository to a GPU host.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfhe_b200.so")
CLI = os.path.join(PKG, "packed_b200")
ROOT = os.path.dirname(PKG)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _host_cxx() -> str:
    # The image's default $CXX wrapper lacks some runtime specs; prefer the
    # system g++ when present.
    for c in ("/usr/bin/g++", os.environ.get("CXX"), shutil.which("g++")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("no host C++ compiler")


def _flags(extra_ptxas: bool) -> list[str]:
    f = ARCH + [
        "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-O2", "-ccbin", _host_cxx(),
        "-I", CSRC, "-I", os.path.join(ROOT, "include"),
    ]
    if extra_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    deps = [src] + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) \
        + glob.glob(os.path.join(ROOT, "include", "*.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [_nvcc(), "-c", src, "-o", obj] + _flags(verbose)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [_nvcc(), "-shared", "-o", LIB] + objs + ARCH + ["-ccbin", _host_cxx(), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    _build_cli()
    return LIB


def _build_cli() -> None:
    """packed_b200: the command-line drop-in for the reference's packed executor."""
    src = os.path.join(CSRC, "packed_main.cpp")
    hdr = os.path.join(ROOT, "include", "fhe_b200.h")
    if os.path.exists(CLI) and os.path.getmtime(CLI) >= max(os.path.getmtime(p) for p in (src, hdr, LIB)):
        return
    cmd = [_host_cxx(), "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), src, "-o", CLI,
           "-L", PKG, "-lfhe_b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"packed_b200 link failed:\n{r.stdout}\n{r.stderr}")


if __name__ == "__main__":
    import sys
    print(build(verbose="-v" in sys.argv))
