"""ctypes binding of libgnnb200.so (the C ABI declared in include/gnn_b200.h).

The library is the product; this module only declares prototypes, turns a
non-zero gnn_status into ``RuntimeError(<gnn_last_error()>)`` (the exception
type a TORCH_CHECK failure raises in the reference) and fails loudly when the
library has not been built: there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("GNNB200_LIB", _PKG / "libgnnb200.so"))

GNN_OK = 0
GNN_ERR_UNSUPPORTED = 3
GNN_AGG_GCN, GNN_AGG_SUM, GNN_AGG_MEAN, GNN_AGG_MEAN_RECIPROCAL = 0, 1, 2, 3
GNN_INDEX_INT32, GNN_INDEX_INT64 = 0, 1
GNN_PRECISION_TF32, GNN_PRECISION_FP32 = 0, 1

_lib = None
_lock = threading.Lock()


class gnn_pointer_info(ctypes.Structure):
    _fields_ = [
        ("memory_type", ctypes.c_int),
        ("device", ctypes.c_int),
        ("is_managed", ctypes.c_int),
        ("is_host_mapped", ctypes.c_int),
        ("pageable_access", ctypes.c_int),
        ("device_pointer", ctypes.c_void_p),
    ]


_vp, _i64, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes)
PROTOTYPES: dict[str, tuple[object, list[object]]] = {
    "gnn_version": (_i32, []),
    "gnn_last_error": (ctypes.c_char_p, []),
    "gnn_status_string": (ctypes.c_char_p, [_i32]),
    "gnn_config_set_int": (_i32, [ctypes.c_char_p, _i64]),
    "gnn_config_get_int": (_i32, [ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "gnn_kernel_launches": (ctypes.c_uint64, []),
    "gnn_gemm_uses_tensor_cores": (_i32, [_i64, _i64, _i64]),
    "gnn_device_status": (_i32, [_i32, ctypes.POINTER(_i32)]),
    "gnn_spmm_workspace_bytes": (_sz, [_i64, _i64]),
    "gnn_spmm_schedule_workspace_bytes": (_sz, [_i64, _i64]),
    "gnn_spmm_long_row_threshold": (_i64, [_i64, _i64]),
    "gnn_spmm_gcn_partition_forward": (
        _i32, [_vp, _i32, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_gcn_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_gcn_hmm_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_gcn_forward_noalloc": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "gnn_spmm_gcn_hmm_optimized_forward": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_stage_feature_pages": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _vp]),
    "gnn_stage_feature_rows": (_i32, [_vp, _i64, _vp, _i64, _i64, _vp]),
    "gnn_spmm_pyg_gcn_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_pyg_gcn_plain_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_pyg_gcn_optimized_forward": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_sum_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "gnn_spmm_mean_forward": (_i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _sz, _vp]),
    "gnn_fused_layer_supported": (_i32, [_i64, _i64, _i64]),
    "gnn_fused_aggregate_linear": (
        _i32, [_vp, _i32, _vp, _vp, _i32, _i64, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _vp, _vp, _i64, _i32, _vp,
               _vp, _i64, _i32, _vp, _vp, _sz, _vp]),
    "gnn_gemm_forward": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "gnn_linear_forward": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "gnn_linear_push_forward": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i32, _vp]),
    "gnn_bias_relu_forward": (_i32, [_vp, _vp, _i64, _i64, _i32, _vp]),
    "gnn_tensor_add_inplace": (_i32, [_vp, _vp, _f32, _i64, _vp]),
    "gnn_relu_inplace": (_i32, [_vp, _i64, _vp]),
    "gnn_managed_alloc": (_i32, [_sz, _i32, ctypes.POINTER(_vp)]),
    "gnn_managed_free": (_i32, [_vp, _i32]),
    "gnn_hmm_supported": (_i32, [_i32, ctypes.POINTER(_i32)]),
    "gnn_copy_host_to_managed": (_i32, [_vp, _vp, _sz]),
    "gnn_prefetch": (_i32, [_vp, _sz, _sz, _sz, _i32, _i32, _vp]),
    "gnn_advise_preferred_location": (_i32, [_vp, _sz, _i32, _i32]),
    "gnn_advise_accessed_by": (_i32, [_vp, _sz, _i32, _i32]),
    "gnn_advise_read_mostly": (_i32, [_vp, _sz, _i32, _i32]),
    "gnn_pointer_info_query": (_i32, [_vp, ctypes.POINTER(gnn_pointer_info)]),
    "gnn_device_accessible_ptr": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "gnn_csr_build_workspace_bytes": (_sz, [_i64, _i64, _i32]),
    "gnn_csr_build": (_i32, [_vp, _vp, _i64, _i64, _i32, _vp, _i32, _vp, _i64, ctypes.POINTER(_i64),
                             ctypes.POINTER(_i64), _vp, _sz, _vp]),
    "gnn_csr_deg_inv_sqrt": (_i32, [_vp, _i32, _i64, _vp, _i64, _vp, _vp]),
    "gnn_csr_edge_weight": (_i32, [_vp, _i32, _vp, _vp, _i64, _vp, _vp]),
    "gnn_locality_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "gnn_locality_page_schedule": (
        _i32, [_vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp,
               ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), _vp, _sz, _vp]),
    "gnn_locality_count_histogram": (_i32, [_vp, _i64, _vp, _i64, _vp]),
    "gnn_locality_coaccess_permutation": (
        _i32, [_vp, _i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _sz, _vp]),
    "gnn_locality_hot_partition": (
        _i32, [_vp, _i64, _i64, _i32, _vp, ctypes.c_double, ctypes.c_double, _i64, _vp, _vp, _vp, _vp,
               ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64), _vp, _sz,
               _vp]),
    "gnn_permute_edges": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _sz, _vp]),
    "gnn_peer_alloc": (_i32, [_sz, _i32, ctypes.POINTER(_vp)]),
    "gnn_peer_free": (_i32, [_vp, _i32]),
    "gnn_ipc_handle_bytes": (_sz, []),
    "gnn_ipc_get_handle": (_i32, [_vp, _vp, _sz]),
    "gnn_ipc_open": (_i32, [_vp, _sz, _i32, ctypes.POINTER(_vp)]),
    "gnn_ipc_close": (_i32, [_vp, _i32]),
    "gnn_can_access_peer": (_i32, [_i32, _i32, ctypes.POINTER(_i32)]),
    "gnn_copy_async": (_i32, [_vp, _vp, _sz, _vp]),
    "gnn_peer_push": (_i32, [_vp, ctypes.POINTER(_vp), _i32, _sz, _i32, _vp]),
    "gnn_peer_push_rows": (_i32, [_vp, ctypes.POINTER(_vp), _i32, _vp, ctypes.POINTER(_i64), _i64, _i64, _i32, _vp]),
}


def lib():
    """Load libgnnb200.so once; raise if it is missing (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"libgnnb200.so not found at {LIB_PATH}; build it with `python gnn_cuda_b200/build.py` "
                    "(or __graft_entry__.build())")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().gnn_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status != GNN_OK:
        msg = last_error() or lib().gnn_status_string(status).decode()
        raise RuntimeError(f"{what}: {msg}" if what and not msg else msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def config_set(name: str, value: int) -> None:
    check(lib().gnn_config_set_int(name.encode(), int(value)), name)


def config_get(name: str) -> int:
    v = ctypes.c_int64(0)
    check(lib().gnn_config_get_int(name.encode(), ctypes.byref(v)), name)
    return int(v.value)


def exported_symbols() -> list[str]:
    return sorted(PROTOTYPES)
