"""Per-phase timing with the reference's API and report format
(GNN_cuda_common/phase_summary.py:11-81).

Difference from the reference: a CUDA phase records a pair of events on the
current stream and returns immediately; durations are resolved when they are
read (``total_ns``, ``iteration_values``, the report). The reference called
``end.synchronize()`` after every phase, which serialised the whole forward.
"""
from __future__ import annotations

import contextlib
import time
from collections import defaultdict

import torch


class PhaseSummary:
    def __init__(self, device: torch.device):
        self.device = device
        self._totals_ns: dict[str, float] = defaultdict(float)
        self._pending: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self._iterations: list[dict] = []

    @contextlib.contextmanager
    def measure(self, key: str, *, use_cuda_events: bool = True):
        if use_cuda_events and self.device.type == "cuda":
            stream = torch.cuda.current_stream(self.device)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            try:
                yield
            finally:
                end.record(stream)
                self._pending.append((key, start, end))
            return
        t0 = time.perf_counter()
        try:
            yield
        finally:
            self._totals_ns[key] += (time.perf_counter() - t0) * 1e9

    def _collect(self, events) -> dict[str, float]:
        sums: dict[str, float] = defaultdict(float)
        for key, start, end in events:
            end.synchronize()
            ns = float(start.elapsed_time(end)) * 1e6
            sums[key] += ns
            self._totals_ns[key] += ns
        return sums

    def _resolve(self) -> None:
        for it in self._iterations:
            if it["values"] is None:
                sums = self._collect(it["events"])
                it["values"] = {k: sums.get(k, 0.0) for k in it["keys"]}
                it["events"] = []
        if self._pending:
            self._collect(self._pending)
            self._pending = []

    def total_ns(self, key: str) -> float:
        self._resolve()
        return float(self._totals_ns.get(key, 0.0))

    def avg_ns(self, key: str, *, iters: int) -> float:
        return self.total_ns(key) / float(iters) if iters > 0 else 0.0

    def record_iteration(self, keys: tuple[str, ...]) -> None:
        """Close an iteration: the phases measured since the previous call belong to it."""
        self._iterations.append({"events": self._pending, "keys": tuple(keys), "values": None})
        self._pending = []

    def iteration_values(self, key: str) -> list[float]:
        self._resolve()
        return [float(it["values"].get(key, 0.0)) for it in self._iterations]

    def reset(self, *, preserve: tuple[str, ...] = ("graph_prep",)) -> None:
        self._resolve()
        kept = {k: self._totals_ns[k] for k in preserve if k in self._totals_ns}
        self._totals_ns.clear()
        self._totals_ns.update(kept)
        self._iterations.clear()


def print_summary_report(summary: PhaseSummary, *, iters: int, infer_avg_ns: float) -> None:
    spmm_avg = summary.avg_ns("spmm", iters=iters)
    print("Summary Report:")
    print(f"spmm, {spmm_avg:.3f}")
    spmm_iters = summary.iteration_values("spmm")
    if spmm_iters:
        print("SpMM Iteration Report:")
        for idx, value in enumerate(spmm_iters, start=1):
            print(f"iter_{idx}, {value:.3f}")
