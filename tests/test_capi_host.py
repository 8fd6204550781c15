"""The C-ABI library on a machine without a GPU: it loads, exports every symbol
that include/gnn_b200.h declares, and rejects bad arguments with the right
status codes before touching the device. Also the Python-layer checks that
mirror the reference's TORCH_CHECK messages."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from gnn_cuda_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]


def _header_functions() -> list[str]:
    text = (ROOT / "include" / "gnn_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gnn_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(N.LIB_PATH))
    names = _header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_prototypes_cover_header():
    assert set(_header_functions()) == set(N.PROTOTYPES)


def test_version_and_status_strings():
    assert N.lib().gnn_version() >= 100
    assert N.lib().gnn_status_string(0) == b"ok"
    assert N.lib().gnn_status_string(7) == b"workspace error"


def test_invalid_arguments_rejected_without_device():
    L = N.lib()
    rc = L.gnn_spmm_sum_forward(None, 0, None, None, None, -1, 0, 4, None, 0, None)
    assert rc == 1 and "must be >= 0" in N.last_error()
    rc = L.gnn_spmm_sum_forward(None, 5, None, None, None, 3, 0, 4, None, 0, None)
    assert rc == 1 and "int32 or int64" in N.last_error()
    rc = L.gnn_spmm_sum_forward(None, 0, None, None, None, 3, 0, 4, None, 0, None)
    assert rc == 2 and "row_ptr" in N.last_error()
    rc = L.gnn_spmm_sum_forward(None, 0, None, None, None, 3, 1 << 33, 4, None, 0, None)
    assert rc == 1 and "int64 row_ptr" in N.last_error()
    # empty problems are valid no-ops
    assert L.gnn_spmm_sum_forward(None, 0, None, None, None, 0, 0, 4, None, 0, None) == 0
    assert L.gnn_gemm_forward(None, None, None, 0, 5, 5, 0, None) == 0
    assert L.gnn_gemm_forward(None, None, None, 4, 5, 5, 9, None) == 1
    rc = L.gnn_spmm_gcn_hmm_optimized_forward(None, 0, None, None, None, None, None, 0, None, 4, 0, 4, None, 0, None)
    assert rc == 2 and "row_schedule must be CUDA" in N.last_error()
    assert L.gnn_stage_feature_rows(None, 3, None, 4, 2, None) == 1
    assert "out rows must be <= x rows" in N.last_error()
    assert L.gnn_prefetch(None, 8, 4, 10, 0, 0, None) == 1
    assert "exceeds tensor byte size" in N.last_error()


def test_workspace_size_query():
    L = N.lib()
    assert L.gnn_spmm_workspace_bytes(0, 0) == 256
    small = L.gnn_spmm_workspace_bytes(1000, 5000)
    big = L.gnn_spmm_workspace_bytes(2_449_029, 64_308_169)
    assert 256 < small < big < 16 * 2**20


def test_config_knobs():
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", 64)
    assert N.config_get("spmm.long_row_threshold") == 64
    N.config_set("spmm.long_row_threshold", old)
    with pytest.raises(RuntimeError, match="unknown config key"):
        N.config_set("nope", 1)
    with pytest.raises(RuntimeError, match=r"\[4, 16\]"):
        N.config_set("spmm.long_row_warps", 64)


@pytest.mark.parametrize("name,default,good,bad", [
    ("spmm.long_row_threshold", 0, [0, 1, 8192], [-1]),
    ("spmm.long_row_warps", 16, [4, 8, 16], [3, 17]),
    ("spmm.kernel", 1, [0, 1, 2], [-1, 3]),
    ("spmm.schedule", 3, [0, 1, 2, 3], [-1, 4]),
    ("spmm.schedule_window", 2048, [1024, 4096, 2**30], [1023, 2**30 + 1]),
    ("gemm.stages", 0, [0, 2, 5, 8], [1, 9, -1]),
])
def test_config_knob_ranges(name, default, good, bad):
    """Every tuning knob: its default, accepted values, and a refusal that leaves the value unchanged."""
    old = N.config_get(name)
    assert old == default
    try:
        for v in good:
            N.config_set(name, v)
            assert N.config_get(name) == v
        N.config_set(name, default)
        for v in bad:
            with pytest.raises(RuntimeError, match=name.replace(".", r"\.")):
                N.config_set(name, v)
            assert N.config_get(name) == default
    finally:
        N.config_set(name, old)


def test_python_checks_match_reference_messages():
    from gnn_cuda_b200.GNN_cuda_common import agg_ops, gcn_ops
    rp = torch.zeros(3, dtype=torch.int32)
    ci = torch.zeros(0, dtype=torch.int32)
    x = torch.zeros(2, 4)
    with pytest.raises(RuntimeError, match="out must be CUDA"):
        agg_ops.spmm_sum_forward_(rp, ci, x, torch.zeros(2, 4))
    with pytest.raises(RuntimeError, match="out must be CUDA"):
        gcn_ops.spmm_gcn_forward_(rp, ci, torch.ones(2), x, torch.zeros(2, 4))
    with pytest.raises(RuntimeError, match="out must be CUDA"):
        agg_ops.gemm_forward_(x, torch.zeros(4, 3), torch.zeros(2, 3))


def test_allocator_modes():
    from gnn_cuda_b200.GNN_cuda_common import allocator as A
    assert A.normalize_memory_mode("managed", allow_hmm=False) == "uvm"
    assert A.normalize_memory_mode("torch_cuda", allow_hmm=True) == "device"
    with pytest.raises(ValueError, match="'hmm' is graph-only"):
        A.normalize_memory_mode("hmm", allow_hmm=False)
    with pytest.raises(ValueError, match="Unsupported memory_mode"):
        A.normalize_memory_mode("bogus", allow_hmm=True)
    assert A.prefers_hmm_spmm("device", "hmm") and not A.prefers_hmm_spmm("uvm", "device")
    with pytest.raises(ValueError, match="requires a CUDA device"):
        A.managed_empty((2, 2), dtype=torch.float32, device=torch.device("cpu"))


def test_locality_arguments_rejected_without_device():
    L = N.lib()
    page = L.gnn_locality_page_schedule
    # num_nodes must be >= 1; top-k lists bounded; required outputs non-NULL
    rc = page(None, 0, None, 0, 0, 8, 64, 4, 8, 16, 4, None, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 1 and "num_nodes" in N.last_error()
    rc = page(None, 0, None, 10, 0, 8, 64, 4, 8, 16, 0, None, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 1 and "signature_topk" in N.last_error()
    rc = page(None, 0, None, 10, 0, 8, 64, 4, 8, 16, 4, None, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 2 and "NULL" in N.last_error()
    rc = L.gnn_locality_coaccess_permutation(None, 0, None, 10, 1 << 33, None, 256, 4, None, None, None, 0, None)
    assert rc == 1 and "num_entries" in N.last_error()
    cut = [ctypes.c_int64(0) for _ in range(4)]
    rc = L.gnn_locality_hot_partition(None, 0, 0, 1, None, 0.8, 0.25, 256, None, None, None, None,
                                      *[ctypes.byref(c) for c in cut], None, 0, None)
    assert rc == 1 and "num_nodes" in N.last_error()
    assert L.gnn_locality_workspace_bytes(10, 10, 5000) == 0
    assert L.gnn_locality_count_histogram(None, 0, None, 0, None) == 1
    assert L.gnn_permute_edges(None, None, 0, None, 5, None, None, None, 0, None) == 0
    assert L.gnn_permute_edges(None, None, 4, None, 5, None, None, None, 0, None) == 2


def test_um_profiler_library_exports_its_header():
    from gnn_cuda_b200.GNN_cuda_common import um_profiler as U
    text = (ROOT / "include" / "gnn_b200_umprof.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(gnn_um_[a-z0-9_]+)\s*\(", text)))
    assert len(names) == 8 and set(names) == set(U.PROTOTYPES)
    lib = ctypes.CDLL(str(U.LIB_PATH))
    assert all(hasattr(lib, n) for n in names)
    # argument checks need no device
    out = U.gnn_um_totals()
    assert U.lib().gnn_um_profiler_totals(5, 1, 0, 0, ctypes.byref(out)) == 1
    assert U.lib().gnn_um_profiler_totals(0, 0, 0, 0, None) == 2
    assert U.lib().gnn_um_profiler_totals(0, 0, 0, 0, ctypes.byref(out)) == 0 and out.records == 0
