#!/usr/bin/env python3
"""Compile the reference's own CUDA aggregation kernels from source into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY. The compiled modules are the GPU-side pin for the
oracle: on a B200 the ``-m gpu`` tests call them on the same seeded tensors as
this repository's kernels and as the C oracle, and check that all three agree
bit for bit on rows that are accumulated in CSR order.

Recipe (mirrors the reference's own JIT loader, ``GNN_cuda_common/loader.py:48-59``):
the sources are compiled exactly where they lie under the reference checkout,
with ``-O3 -std=c++17`` and the architecture list the reference would pick on a
B200 (compute capability 10.0, ``loader.py:42-44``). Nothing is copied into
this repository; the build products go only to ``oracle/_ref/`` (git-ignored,
but shipped to the GPU machine with the rest of the tree).

Usage:  python oracle/build_ref.py [--reference DIR] [--jobs 3]
(DIR defaults to $GNN_REFERENCE_ROOT, else a ``reference`` directory beside this repository.)
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys
from concurrent.futures import ProcessPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"

# module name -> sources (relative to GNN_cuda_common/native/ in the reference)
MODULES = {
    "ref_gcn_ops": ["gcn_ops.cpp", "gcn_ops.cu"],
    "ref_pyg_gcn_ops": ["pyg_gcn_ops.cpp", "pyg_gcn_ops.cu"],
    "ref_agg_ops": ["agg_ops.cpp", "agg_ops.cu"],
}


def _build_one(args: tuple[str, list[str], str]) -> str:
    name, sources, native_dir = args
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", "2")
    from torch.utils.cpp_extension import load

    build_dir = OUT / "build" / name
    build_dir.mkdir(parents=True, exist_ok=True)
    load(
        name=name,
        sources=[str(Path(native_dir) / s) for s in sources],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "-std=c++17"],
        build_directory=str(build_dir),
        verbose=False,
    )
    so = build_dir / f"{name}.so"
    dst = OUT / f"{name}.so"
    shutil.copy2(so, dst)
    return str(dst)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GNN_REFERENCE_ROOT", str(HERE.parent.parent / "reference")))
    ap.add_argument("--jobs", type=int, default=3)
    args = ap.parse_args()
    native_dir = Path(args.reference) / "GNN_cuda_common" / "native"
    if not native_dir.is_dir():
        print(f"reference sources not found at {native_dir}; nothing built", file=sys.stderr)
        return 1
    OUT.mkdir(parents=True, exist_ok=True)
    work = [(n, s, str(native_dir)) for n, s in MODULES.items()]
    with ProcessPoolExecutor(max_workers=max(1, args.jobs)) as ex:
        for path in ex.map(_build_one, work):
            print("built", path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
