#!/usr/bin/env python3
"""Build ``libgnnb200.so`` in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in
parallel, only when its source or a header changed) and linked into
``gnn_cuda_b200/libgnnb200.so``. The library links the CUDA runtime
statically and has no PyTorch dependency: it is the C ABI declared in
``include/gnn_b200.h``.

Numerics flags are the CUDA defaults on purpose: IEEE division and square
root, no flush-to-zero, and fused multiply-add only where the source asks for
it (the kernels use explicit __fmaf_rn / __fadd_rn / __fmul_rn intrinsics).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build" / "gnnb200"
LIB = PKG / "libgnnb200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    deps = _headers() + [Path(__file__)]
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_info or _stale(obj, src, deps):
            cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd: list[str]) -> tuple[list[str], subprocess.CompletedProcess]:
        return cmd, subprocess.run(cmd, capture_output=True, text=True)

    failed = []
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cmd, res in ex.map(run, jobs):
            if verbose or ptxas_info or res.returncode != 0:
                sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            if res.returncode != 0:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError(f"nvcc failed for: {failed}")

    if jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            raise RuntimeError("link of libgnnb200.so failed")
        os.replace(tmp, LIB)
    build_umprof()
    return LIB


UMPROF_SRC = PKG / "csrc_prof" / "um_profiler.cpp"
UMPROF_LIB = PKG / "libgnnb200_umprof.so"


def _cuda_root() -> Path:
    return Path(_nvcc()).resolve().parent.parent


def build_umprof(force: bool = False) -> Path:
    """libgnnb200_umprof.so: the CUPTI unified-memory counter library (host code
    only, linked against the toolkit's libcupti with an rpath to it)."""
    deps = [UMPROF_SRC, INCLUDE / "gnn_b200_umprof.h", INCLUDE / "gnn_b200.h", Path(__file__)]
    if not force and UMPROF_LIB.exists() and all(p.stat().st_mtime <= UMPROF_LIB.stat().st_mtime for p in deps):
        return UMPROF_LIB
    cuda = _cuda_root()
    libdir = cuda / "lib64"
    tmp = UMPROF_LIB.with_suffix(".so.tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-I{INCLUDE}", f"-I{cuda / 'include'}", str(UMPROF_SRC), "-o", str(tmp), f"-L{libdir}", "-lcupti",
           f"-Wl,-rpath,{libdir}", "-Wl,--exclude-libs,ALL", "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        raise RuntimeError("build of libgnnb200_umprof.so failed")
    os.replace(tmp, UMPROF_LIB)
    return UMPROF_LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print register/smem usage per kernel")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, ptxas_info=args.ptxas_info, force=args.force))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
