"""Unified-memory counters through CUPTI (libgnnb200_umprof.so), the nsys-free
replacement of run/profile_spmm_migration.py's measurement.

Each case runs in a fresh subprocess so that the counters are switched on
before the process creates its CUDA context, as the profiler requires.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

_TOUCH = r'''
import json, sys, torch
sys.path.insert(0, sys.argv[1])
from gnn_cuda_b200.GNN_cuda_common.um_profiler import UMProfiler
from gnn_cuda_b200.GNN_cuda_common import allocator as A
prof = UMProfiler().start()
dev = torch.device("cuda", 0)
out = {}
for prefetch in (False, True):
    n = 16 * 2**20  # 64 MiB of float32
    host = torch.arange(n, dtype=torch.float32)
    t = A.managed_empty((n,), dtype=torch.float32, device=dev)
    A.load_allocator_module().copy_cpu_to_managed_(t, host)  # pages start on the host
    if prefetch:
        A.prefetch_managed(t, location="cuda", device=dev)
    s = float(t.sum().item())  # the GPU reads every page
    torch.cuda.synchronize()
    prof.flush()
    lo = t.data_ptr(); hi = lo + n * 4
    out["prefetch" if prefetch else "touch"] = dict(prof.totals((lo, hi)), ok=(s == float(host.sum().item())),
                                                    kinds=UMProfiler.enabled_kinds())
    del t
prof.stop()
print(json.dumps(out))
'''


def test_um_counters_see_migrations_and_faults():
    res = subprocess.run([sys.executable, "-c", _TOUCH, str(ROOT)], capture_output=True, text=True, timeout=300)
    if "UM_PROFILING_NOT_SUPPORTED" in res.stderr or "nvidia-uvm-tools" in res.stderr:
        pytest.skip("unified-memory counters are not available on this system")
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    size = 64 * 2**20
    touch, pre = out["touch"], out["prefetch"]
    assert touch["ok"] and pre["ok"]
    # first touch on the GPU migrates the pages host -> device through page faults
    assert touch["kinds"] >= 3, "GPU page-fault counters are needed for the migration report"
    assert touch["htod_bytes"] >= 0.9 * size and touch["gpu_page_faults"] > 0
    # a prefetch migrates them ahead of the kernel: same bytes, (almost) no faults
    assert pre["htod_bytes"] >= 0.9 * size
    assert pre["gpu_page_faults"] < 0.1 * touch["gpu_page_faults"] + 1
    assert touch["dropped_records"] == 0


def _summary(text: str) -> dict:
    vals = {}
    for line in text.splitlines():
        if "," in line:
            k, v = line.split(",", 1)
            try:
                vals[k.strip()] = float(v)
            except ValueError:
                pass
    return vals


@pytest.mark.parametrize("ft_matrix,prefetch,host_alloc", [("uvm", 0, 0.0), ("uvm", 1, 0.0), ("uvm", 1, 20.0)])
def test_profile_spmm_migration_reports_feature_range_traffic(tmp_path, ft_matrix, prefetch, host_alloc):
    from gnn_cuda_b200 import synth
    from gnn_cuda_b200.GNN_cuda_common.npz_utils import save_graph_npz
    n = 60_000
    u, v = synth.rmat_undirected(n, n * 8, seed=81)
    s, d = synth.symmetrize(u, v)
    save_graph_npz(str(tmp_path / "tiny.npz"), s.numpy(), d.numpy(), n)
    cmd = [sys.executable, "-m", "gnn_cuda_b200.run.profile_spmm_migration", "--dataset", "tiny", "--data_root",
           str(tmp_path), "--ft_matrix", ft_matrix, "--prefetch", str(prefetch), "--ft_host_alloc", str(host_alloc),
           "--dim", "256", "--iters", "3", "--output_dir", str(tmp_path / "out")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert res.returncode == 0, res.stderr[-3000:]
    vals = _summary(res.stdout)
    feature_bytes = n * 256 * 4
    assert vals["spmm_ns"] > 0
    if "nvidia-uvm-tools" in res.stderr:
        # no unified-memory counters on this system: the SpMM time is still reported, the fault
        # count is nan, and the bytes come from NVML's host-link counters (the whole device's
        # PCIe bytes per iteration of the measured loop) when NVML answers, else nan
        assert np.isnan(vals["GPU_faults"])
        assert np.isnan(vals["HtoD_bytes"]) or vals["HtoD_bytes"] >= 0
    else:
        assert vals["HtoD_bytes"] >= 0.5 * feature_bytes  # the features are initialised on the host side
        if prefetch == 0:
            assert vals["GPU_faults"] > 0
    summaries = list((tmp_path / "out").glob("*_summary.txt"))
    assert len(summaries) == 1 and "HtoD_bytes" in summaries[0].read_text()
