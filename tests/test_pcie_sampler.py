"""The NVML host-link fallback of the migration profiler, on the host with a fake reader.

Where CUPTI's unified-memory counters are unavailable, run/profile_spmm_migration.py
reports HtoD/DtoH bytes as the integral of NVML's PCIe RX/TX throughput (KB/s)
over the measured loop; the integration is checked here against a constant rate.
"""
import time

from gnn_cuda_b200.GNN_cuda_common.um_profiler import PcieSampler


def test_constant_rate_integrates_to_rate_times_time():
    s = PcieSampler(0, period_s=0.005, read=lambda: (2048.0, 512.0)).start()
    t0 = time.perf_counter()
    time.sleep(0.25)
    s.stop()
    dt = time.perf_counter() - t0
    assert s.samples >= 10
    # every sample covers the time since the previous one: the total is within one period of rate x time
    assert abs(s.rx_bytes - 2048 * 1024 * dt) <= 2048 * 1024 * 0.05
    assert abs(s.tx_bytes / s.rx_bytes - 0.25) < 1e-9


def test_restart_clears_totals():
    s = PcieSampler(0, period_s=0.005, read=lambda: (100.0, 100.0)).start()
    time.sleep(0.05)
    s.stop()
    s.start()
    s.stop()
    assert s.rx_bytes < 100 * 1024 * 0.05
