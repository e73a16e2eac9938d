"""Build the native libraries of jstorch_b200 in-tree (no JIT cache).

    python -m jstorch_b200.build            # build what is out of date
    python -m jstorch_b200.build --force    # rebuild everything
    python -m jstorch_b200.build --ptxas-v  # print register / spill / smem use

Outputs (git-ignored, shipped with the source tree):
    jstorch_b200/libjstorch_gemm.so   the C-ABI GEMM library (include/jstorch_gemm.h, jstorch_conv.h)
    jstorch_b200/_core*.so            the host core (Tensor / GradTensor), Python extension
    jstorch_b200/libjstorch_dist.so   the NCCL sharded GEMMs (include/jstorch_dist.h)

Every CUDA source is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); nvcc cross-compiles on a host
without a GPU.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = ROOT / "include"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", f"{CUDA_HOME}/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
           "--expt-relaxed-constexpr", "-DNDEBUG", f"-I{INCLUDE}"] + ARCH

GEMM_SOURCES = ["gemm_api.cu", "gemm_ffma.cu", "gemm_tc.cu", "splitk.cu", "conv.cu", "gru.cu", "hostio.cu", "profile.cu"]
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
    headers = [CSRC / h for h in GEMM_HEADERS] + [INCLUDE / "jstorch_gemm.h", INCLUDE / "jstorch_conv.h", INCLUDE / "jstorch_rnn.h"]
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


CORE = CSRC / "core"
CORE_CPP = ["tensor.cpp", "autograd.cpp", "allocator.cpp", "compiled.cpp", "binding.cpp"]
CORE_CU = ["kernels.cu"]
CORE_HEADERS = ["tensor.h", "autograd.h", "allocator.h", "compiled.h", "core_kernels.h"]
CORE_EXT = PKG / ("_core" + sysconfig.get_config_var("EXT_SUFFIX"))
CXX = os.environ.get("CXX", "g++")


def build_core(force: bool = False, verbose: bool = False) -> Path:
    """The host core (Tensor / GradTensor) as the Python extension _core,
    linked against libjstorch_gemm.so (found next to it at run time)."""
    import pybind11

    BUILD.mkdir(exist_ok=True)
    headers = [CORE / h for h in CORE_HEADERS] + [INCLUDE / "jstorch_gemm.h"]
    objs = []
    incs = [f"-I{INCLUDE}", f"-I{CUDA_HOME}/include", f"-I{sysconfig.get_paths()['include']}",
            f"-I{pybind11.get_include()}"]
    for src in CORE_CPP:
        s = CORE / src
        o = BUILD / ("core_" + s.stem + ".o")
        objs.append(o)
        if force or not _newer(o, [s] + headers + [Path(__file__)]):
            _run([CXX, "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", *incs, "-c", str(s), "-o",
                  str(o)], verbose)
    for src in CORE_CU:
        s = CORE / src
        o = BUILD / ("core_" + s.stem + ".o")
        objs.append(o)
        if force or not _newer(o, [s] + headers + [Path(__file__)]):
            _run([NVCC, *NVFLAGS, "-c", str(s), "-o", str(o)], verbose)
    if force or not _newer(CORE_EXT, objs + [GEMM_LIB]):
        tmp = CORE_EXT.with_suffix(".tmp")
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), f"-L{PKG}", "-ljstorch_gemm",
              "-Xlinker", "-rpath,$ORIGIN"], verbose)
        os.replace(tmp, CORE_EXT)
    return CORE_EXT


DIST_SOURCES = ["dist.cu", "symm.cu", "reg.cu"]
DIST_LIB = PKG / "libjstorch_dist.so"


def build_dist(force: bool = False, verbose: bool = False) -> Path:
    """libjstorch_dist.so: the NCCL sharded GEMMs (include/jstorch_dist.h),
    linked against libjstorch_gemm.so and the system NCCL."""
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in GEMM_HEADERS + ["dist_internal.h"]] + [INCLUDE / "jstorch_gemm.h",
                                                                         INCLUDE / "jstorch_dist.h"]
    objs = []
    for src in DIST_SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or not _newer(o, [s] + headers + [Path(__file__)]):
            _run([NVCC, *NVFLAGS, "-c", str(s), "-o", str(o)], verbose)
    if force or not _newer(DIST_LIB, objs + [GEMM_LIB]):
        tmp = DIST_LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), f"-L{PKG}", "-ljstorch_gemm", "-lnccl",
              "-Xlinker", "-rpath,$ORIGIN"], verbose)
        os.replace(tmp, DIST_LIB)
    return DIST_LIB


def build_all(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> None:
    build_gemm(force=force, ptxas_v=ptxas_v, verbose=verbose)
    build_core(force=force, verbose=verbose)
    build_dist(force=force, verbose=verbose)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    build_all(force=a.force, ptxas_v=a.ptxas_v, verbose=a.verbose)
    print(f"built {GEMM_LIB.relative_to(ROOT)} {CORE_EXT.relative_to(ROOT)} {DIST_LIB.relative_to(ROOT)}")


if __name__ == "__main__":
    main()
