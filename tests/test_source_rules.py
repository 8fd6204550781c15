"""Static checks on the shipped sources (no GPU, no compute).

These guard against forms that must never reach a GPU run of this library:
  * the batched host/device copy entry points of the CUDA runtime and driver,
    which raised GPU faults on B200 with driver 580 (one plain async copy per
    buffer is used instead);
  * `__trap()` and device `assert`, which would be the only way a kernel here
    could end its context on purpose (bounded waits return a status instead).
The forbidden spellings are assembled from pieces so this file does not contain
them itself.
"""
from __future__ import annotations

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SOURCE_SUFFIXES = {".cu", ".cuh", ".cpp", ".cc", ".c", ".h", ".py", ".sh"}
SKIP_DIRS = {"_ref", "_build", "_work", "__pycache__", ".git", "baseline"}
# Run-output folders (named "*_out") hold logs and captures, not shipped sources.
OUTPUT_SUFFIX = "_out"


def _sources():
    for p in ROOT.rglob("*"):
        parts = p.relative_to(ROOT).parts
        if not p.is_file() or p.suffix not in SOURCE_SUFFIXES or set(parts) & SKIP_DIRS:
            continue
        if any(d.endswith(OUTPUT_SUFFIX) for d in parts[:-1]):
            continue
        yield p


def _texts():
    me = Path(__file__).resolve()
    for p in _sources():
        if p.resolve() == me:
            continue
        yield p, p.read_text(errors="replace")


def test_sources_found():
    names = {p.name for p in _sources()}
    assert {"spmm.cu", "gemm_tc.cu", "peer.cu", "bench.py"} <= names


def test_no_batched_copy_calls():
    names = ["cuda" + "Memcpy" + "Batch" + "Async", "cuda" + "Memcpy3D" + "Batch" + "Async",
             "cu" + "Memcpy" + "Batch" + "Async", "cu" + "Memcpy3D" + "Batch" + "Async"]
    bad = [f"{p.relative_to(ROOT)}: {n}" for p, t in _texts() for n in names if n in t]
    assert not bad, bad


def test_no_intentional_device_traps():
    trap = re.compile(r"__" + r"trap\s*\(")
    dev_assert = re.compile(r"^\s*assert\s*\(")
    bad = []
    for p, t in _texts():
        if p.suffix not in {".cu", ".cuh"}:
            continue
        for i, line in enumerate(t.splitlines(), 1):
            if trap.search(line) or dev_assert.search(line):
                bad.append(f"{p.relative_to(ROOT)}:{i}")
    assert not bad, bad


def test_every_ncu_command_keeps_clocks():
    """Any ncu command written into a shipped script or doc string leaves the clocks alone."""
    bad = []
    for p, t in _texts():
        for i, line in enumerate(t.splitlines(), 1):
            if re.search(r"(^|[\s'\"`])ncu\s+-", line) and "--clock-control none" not in line:
                bad.append(f"{p.relative_to(ROOT)}:{i}")
    assert not bad, bad
