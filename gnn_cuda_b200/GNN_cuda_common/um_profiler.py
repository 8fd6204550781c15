"""Unified-memory migration counters in-process (CUPTI), in place of nsys.

ctypes binding of ``libgnnb200_umprof.so`` (``include/gnn_b200_umprof.h``).
The reference obtains HtoD/DtoH migration bytes and GPU page faults over the
feature matrix's address range from an nsys SQLite export
(run/profile_spmm_migration.py:303-461); ``UMProfiler.totals`` applies the same
filters to CUPTI's unified-memory counter records collected in this process.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parents[1]
LIB_PATH = Path(os.environ.get("GNNB200_UMPROF_LIB", _PKG / "libgnnb200_umprof.so"))

_lib = None
_lock = threading.Lock()


class gnn_um_totals(ctypes.Structure):
    _fields_ = [
        ("htod_bytes", ctypes.c_double),
        ("dtoh_bytes", ctypes.c_double),
        ("gpu_page_faults", ctypes.c_double),
        ("cpu_page_faults", ctypes.c_double),
        ("thrashing_bytes", ctypes.c_double),
        ("throttling_events", ctypes.c_double),
        ("remote_map_bytes", ctypes.c_double),
        ("records", ctypes.c_uint64),
        ("dropped_records", ctypes.c_uint64),
    ]


PROTOTYPES = {
    "gnn_um_profiler_start": (ctypes.c_int, []),
    "gnn_um_profiler_flush": (ctypes.c_int, []),
    "gnn_um_profiler_stop": (ctypes.c_int, []),
    "gnn_um_profiler_clear": (ctypes.c_int, []),
    "gnn_um_profiler_timestamp": (ctypes.c_uint64, []),
    "gnn_um_profiler_totals": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                              ctypes.POINTER(gnn_um_totals)]),
    "gnn_um_profiler_enabled_kinds": (ctypes.c_int, []),
    "gnn_um_profiler_last_error": (ctypes.c_char_p, []),
}


def lib():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"libgnnb200_umprof.so not found at {LIB_PATH}; build it with "
                                   "`python gnn_cuda_b200/build.py`")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def _check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().gnn_um_profiler_last_error()
        raise RuntimeError(f"{what}: {msg.decode() if msg else status}")


class UMProfiler:
    """Collects CUPTI unified-memory counter records for this process.

    Start it before the first CUDA call where possible. ``totals`` sums the
    records over an address range and a CUPTI time window with the reference's
    rules: migrations whose byte range overlaps the address range, faults whose
    address lies inside it.
    """

    def start(self) -> "UMProfiler":
        _check(lib().gnn_um_profiler_start(), "gnn_um_profiler_start")
        return self

    @staticmethod
    def enabled_kinds() -> int:
        """Counter kinds collected: 7 = all, 3 = HtoD/DtoH/GPU faults, 2 = HtoD/DtoH."""
        return int(lib().gnn_um_profiler_enabled_kinds())

    def flush(self) -> None:
        _check(lib().gnn_um_profiler_flush(), "gnn_um_profiler_flush")

    def stop(self) -> None:
        _check(lib().gnn_um_profiler_stop(), "gnn_um_profiler_stop")

    def clear(self) -> None:
        _check(lib().gnn_um_profiler_clear(), "gnn_um_profiler_clear")

    @staticmethod
    def timestamp() -> int:
        return int(lib().gnn_um_profiler_timestamp())

    def totals(self, address_range: tuple[int, int] | None = None, window: tuple[int, int] | None = None) -> dict:
        lo, hi = address_range if address_range is not None else (0, 0)
        t0, t1 = window if window is not None else (0, 0)
        out = gnn_um_totals()
        _check(lib().gnn_um_profiler_totals(int(lo), int(hi), int(t0), int(t1), ctypes.byref(out)),
               "gnn_um_profiler_totals")
        return {name: getattr(out, name) for name, _ in gnn_um_totals._fields_}
