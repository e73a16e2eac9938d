"""Build the native libraries of jstorch_b200 in-tree (no JIT cache).

    python -m jstorch_b200.build            # build what is out of date
    python -m jstorch_b200.build --force    # rebuild everything
    python -m jstorch_b200.build --ptxas-v  # print register / spill / smem use

Outputs (git-ignored, shipped with the source tree):
    jstorch_b200/libjstorch_gemm.so   the C-ABI GEMM library (include/jstorch_gemm.h)

Every CUDA source is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); nvcc cross-compiles on a host
without a GPU.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
           "--expt-relaxed-constexpr", "-DNDEBUG", f"-I{INCLUDE}"] + ARCH

GEMM_SOURCES = ["gemm_api.cu", "gemm_ffma.cu", "gemm_tc.cu", "profile.cu"]
GEMM_HEADERS = ["gemm_internal.h", "ptx.cuh"]
GEMM_LIB = PKG / "libjstorch_gemm.so"


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.stdout and verbose:
        print(r.stdout, end="")
    if r.returncode != 0 or (r.stderr and verbose):
        sys.stderr.write(r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}")


def build_gemm(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in GEMM_HEADERS] + [INCLUDE / "jstorch_gemm.h"]
    objs = []
    for src in GEMM_SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or ptxas_v or not _newer(o, [s] + headers + [Path(__file__)]):
            extra = ["-Xptxas", "-v"] if ptxas_v else []
            _run([NVCC, *NVFLAGS, *extra, "-c", str(s), "-o", str(o)], verbose or ptxas_v)
    if force or not _newer(GEMM_LIB, objs):
        tmp = GEMM_LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)], verbose)
        os.replace(tmp, GEMM_LIB)
    return GEMM_LIB


def build_all(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> None:
    build_gemm(force=force, ptxas_v=ptxas_v, verbose=verbose)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    build_all(force=a.force, ptxas_v=a.ptxas_v, verbose=a.verbose)
    print(f"built {GEMM_LIB.relative_to(ROOT)}")


if __name__ == "__main__":
    main()
