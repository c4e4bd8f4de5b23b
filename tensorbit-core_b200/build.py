"""Builds the B200 pruning library and CLI in-tree.

  python tensorbit-core_b200/build.py            # lib/libtb_b200.so (+ bin/ when sources exist)
  python tensorbit-core_b200/build.py --verbose  # also print ptxas register/spill reports

CUDA sources are compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with round-to-nearest FP and no
fast-math, so the kernels keep the reference's IEEE float results; host C++ is
compiled by g++ with -ffp-contract=off for the same reason.  Objects are
rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB_DIR = os.path.join(PKG, "lib")
BIN_DIR = os.path.join(PKG, "bin")
LIB = os.path.join(LIB_DIR, "libtb_b200.so")
INCLUDES = [os.path.join(ROOT, "include"), CSRC, os.path.join(PKG, "include")]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off",
                     "--expt-relaxed-constexpr", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
                     "-fmad=false"]
CXX_FLAGS = ["-std=c++20", "-O2", "-fPIC", "-ffp-contract=off", "-Wall"]


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(ROOT, "include", "*.h"))
            + glob.glob(os.path.join(PKG, "include", "tensorbit", "core", "*.hpp")))


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd: list[str], verbose: bool) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")
    if verbose and (r.stdout or r.stderr):
        sys.stdout.write(r.stdout + r.stderr)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _deps()):
        return obj
    inc = [f"-I{d}" for d in INCLUDES]
    if src.endswith(".cu"):
        extra = ["-Xptxas", "-v"] if verbose else []
        cmd = [NVCC] + NVCC_FLAGS + extra + inc + ["-c", "-o", obj, src]
    else:
        cmd = [CXX] + CXX_FLAGS + inc + [f"-I{os.path.join(os.path.dirname(NVCC), '..', 'include')}",
                                         "-c", "-o", obj, src]
    _run(cmd, verbose)
    return obj


def build(verbose: bool = False) -> str:
    if not os.path.exists(NVCC) and not shutil.which("nvcc"):
        raise RuntimeError("nvcc not found: the CUDA library cannot be built")
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread"], verbose)
    _build_cli(verbose)
    return LIB


def _build_cli(verbose: bool) -> None:
    """Host C++ programs (tb-prune, the host API test driver) linked to the library."""
    progs = glob.glob(os.path.join(PKG, "cli", "*.cpp"))
    if not progs:
        return
    os.makedirs(BIN_DIR, exist_ok=True)
    inc = [f"-I{d}" for d in INCLUDES]
    for src in progs:
        name = os.path.splitext(os.path.basename(src))[0].replace("_", "-")
        out = os.path.join(BIN_DIR, name)
        if _stale(out, [src, LIB] + _deps()):
            _run([CXX] + CXX_FLAGS + inc + ["-o", out, src, f"-L{LIB_DIR}", "-ltb_b200",
                                            f"-Wl,-rpath,$ORIGIN/../lib", "-lpthread"], verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose))
