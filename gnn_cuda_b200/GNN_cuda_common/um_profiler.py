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


class PcieSampler:
    """Host-link bytes of one GPU over a time window, from NVML's PCIe throughput
    counters (KB/s over 20 ms windows, sampled every `period_s` and integrated).

    The fallback where CUPTI's unified-memory counters are unavailable (no
    /dev/nvidia-uvm-tools): during an aggregation over unified-memory features
    the host-to-device traffic is the feature migration, so the RX bytes stand in
    for the reference's HtoD_bytes — of the whole device rather than of the
    feature range, and without a page-fault count. `read` may be replaced (tests)
    by any callable returning (rx_kb_per_s, tx_kb_per_s)."""

    def __init__(self, device_index: int = 0, period_s: float = 0.02, read=None):
        self.period_s = float(period_s)
        self._read = read
        self._dev = int(device_index)
        self._stop = threading.Event()
        self._thread = None
        self.rx_bytes = 0.0
        self.tx_bytes = 0.0
        self.samples = 0

    def _nvml_reader(self):
        import pynvml
        pynvml.nvmlInit()
        handle = None
        try:
            import torch
            props = torch.cuda.get_device_properties(self._dev)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self._dev)

        def read():
            return (pynvml.nvmlDeviceGetPcieThroughput(handle, pynvml.NVML_PCIE_UTIL_RX_BYTES),
                    pynvml.nvmlDeviceGetPcieThroughput(handle, pynvml.NVML_PCIE_UTIL_TX_BYTES))
        return read

    def start(self) -> "PcieSampler":
        if self._read is None:
            self._read = self._nvml_reader()
        self._stop.clear()
        self.rx_bytes = self.tx_bytes = 0.0
        self.samples = 0

        def loop():
            import time
            last = time.perf_counter()
            while not self._stop.wait(self.period_s):
                now = time.perf_counter()
                rx, tx = self._read()
                self.rx_bytes += float(rx) * 1024.0 * (now - last)
                self.tx_bytes += float(tx) * 1024.0 * (now - last)
                self.samples += 1
                last = now
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
