"""The native operator tables of GNN_cuda, re-implemented over libgnnb200.so.

One Python function per entry of the reference's pybind11 tables
(``GNN_cuda_common/native/agg_ops.cpp:18-36``, ``gcn_ops.cpp:21-32``,
``pyg_gcn_ops.cpp:21-32``, ``uvm_allocator.cpp:21-38``), with the same
arguments, the same input checks (same message text, raised as RuntimeError
like a TORCH_CHECK) and in-place semantics. Each call resolves device-usable
pointers exactly like ``tensor_access.cuh:25-64`` (CUDA tensors directly;
CPU tensors through a mapped-pinned alias or HMM pageable access), then calls
the C ABI on the *current* CUDA stream of the output's device. The reference
launched on the device's default stream; for callers that never change the
current stream the two are the same stream.
"""
from __future__ import annotations

import ctypes
import threading
from types import SimpleNamespace

import torch

from .. import _native as N

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _dev_ptr(t: torch.Tensor | None) -> int | None:
    """Device-usable address of a tensor (tensor_access.cuh:25-64)."""
    if t is None or t.numel() == 0:
        return None
    if t.is_cuda:
        return t.data_ptr()
    _check(t.device.type == "cpu", "Expected CPU or CUDA tensor for device access")
    out = ctypes.c_void_p()
    N.check(N.lib().gnn_device_accessible_ptr(ctypes.c_void_p(t.data_ptr()), ctypes.byref(out)))
    return out.value


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _workspace(device: torch.device, nbytes: int) -> tuple[int, int]:
    """A per-(device, stream) scratch buffer, grown on demand and reused.

    Calls on one stream are ordered, so they can share one workspace.
    """
    if nbytes <= 0:
        return 0, 0
    key = (device.index if device.index is not None else torch.cuda.current_device(), _stream(device))
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
            _workspaces[key] = buf
    return buf.data_ptr(), buf.numel()


def ensure_workspace(device: torch.device, num_nodes: int, num_edges: int) -> None:
    """Allocate the aggregation workspace of the current stream now (e.g. before a
    caller reserves the rest of device memory), so later calls allocate nothing."""
    with torch.cuda.device(device):
        _workspace(device, N.lib().gnn_spmm_schedule_workspace_bytes(int(num_nodes), int(num_edges)))


def _index_type(row_ptr: torch.Tensor) -> int:
    if row_ptr.dtype == torch.int32:
        return N.GNN_INDEX_INT32
    _check(row_ptr.dtype == torch.int64, "row_ptr must be int32")
    return N.GNN_INDEX_INT64


# ---------------------------------------------------------------------------
# shared checks (agg_ops.cu:168-189, gcn_ops.cu:229-258, pyg_gcn_ops.cu:194-223)
# ---------------------------------------------------------------------------

def _check_csr_common(row_ptr, col_ind, x, out, extra: dict[str, torch.Tensor]) -> None:
    _check(out.is_cuda, "out must be CUDA")
    _check(row_ptr.is_contiguous(), "row_ptr must be contiguous")
    _check(col_ind.is_contiguous(), "col_ind must be contiguous")
    for name, t in extra.items():
        _check(t.is_contiguous(), f"{name} must be contiguous")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(out.is_contiguous(), "out must be contiguous")
    _check(row_ptr.dtype in (torch.int32, torch.int64), "row_ptr must be int32")
    _check(col_ind.dtype == torch.int32, "col_ind must be int32")
    for name, t in extra.items():
        _check(t.dtype == torch.float32, f"{name} must be float32")
    _check(x.dtype == torch.float32, "x must be float32")
    _check(out.dtype == torch.float32, "out must be float32")
    _check(x.dim() == 2, "x must be rank-2")
    _check(out.dim() == 2, "out must be rank-2")
    _check(tuple(x.shape) == tuple(out.shape), "x and out must have the same shape")
    _check(row_ptr.dim() == 1, "row_ptr must be rank-1")
    _check(col_ind.dim() == 1, "col_ind must be rank-1")
    for name, t in extra.items():
        _check(t.dim() == 1, f"{name} must be rank-1")
    _check(row_ptr.numel() == x.size(0) + 1, "row_ptr length must be num_nodes + 1")


def _check_optimized(row_schedule, hot_feature_cache, x, hot_node_cutoff: int) -> None:
    """gcn_ops.cu:260-285 / pyg_gcn_ops.cu:225-250."""
    _check(row_schedule is not None and row_schedule.is_cuda, "row_schedule must be CUDA")
    _check(hot_feature_cache is not None and hot_feature_cache.is_cuda, "hot_feature_cache must be CUDA")
    _check(row_schedule.is_contiguous(), "row_schedule must be contiguous")
    _check(hot_feature_cache.is_contiguous(), "hot_feature_cache must be contiguous")
    _check(row_schedule.dtype == torch.int64, "row_schedule must be int64")
    _check(hot_feature_cache.dtype == torch.float32, "hot_feature_cache must be float32")
    _check(row_schedule.dim() == 1, "row_schedule must be rank-1")
    _check(hot_feature_cache.dim() == 2, "hot_feature_cache must be rank-2")
    _check(row_schedule.numel() == x.size(0), "row_schedule length must equal num_nodes")
    _check(hot_node_cutoff >= 1, "hot_node_cutoff must be >= 1")
    _check(hot_node_cutoff <= x.size(0), "hot_node_cutoff must be <= num_nodes")
    _check(hot_feature_cache.size(0) == hot_node_cutoff, "hot_feature_cache row count must equal hot_node_cutoff")
    _check(hot_feature_cache.size(1) == x.size(1), "hot_feature_cache feature dimension must match x")


def _spmm_call(fn_name: str, row_ptr, col_ind, vec, x, out, *extra_args, optimized=None):
    n, f = int(x.size(0)), int(x.size(1))
    nnz = int(col_ind.numel())
    dev = out.device
    with torch.cuda.device(dev):
        rp, ci, vp, xp = _dev_ptr(row_ptr), _dev_ptr(col_ind), _dev_ptr(vec), _dev_ptr(x)
        ws, wsb = _workspace(dev, N.lib().gnn_spmm_schedule_workspace_bytes(n, nnz))
        s = _stream(dev)
        fn = getattr(N.lib(), fn_name)
        if optimized is not None:
            sched, hot, cutoff = optimized
            rc = fn(rp, _index_type(row_ptr), ci, vp, xp, sched.data_ptr(), hot.data_ptr(), int(cutoff),
                    out.data_ptr(), n, nnz, f, ws, wsb, s)
        elif vec is None and fn_name == "gnn_spmm_mean_forward":
            rc = fn(rp, _index_type(row_ptr), ci, xp, out.data_ptr(), n, nnz, f, *extra_args, ws, wsb, s)
        elif vec is None:
            rc = fn(rp, _index_type(row_ptr), ci, xp, out.data_ptr(), n, nnz, f, ws, wsb, s)
        else:
            rc = fn(rp, _index_type(row_ptr), ci, vp, xp, out.data_ptr(), n, nnz, f, ws, wsb, s)
        N.check(rc)


# ---------------------------------------------------------------------------
# gcn_ops table (gcn_ops.cpp:21-32)
# ---------------------------------------------------------------------------

def _gcn_checks(row_ptr, col_ind, deg_inv_sqrt, x, out):
    _check_csr_common(row_ptr, col_ind, x, out, {"deg_inv_sqrt": deg_inv_sqrt})
    _check(deg_inv_sqrt.numel() == x.size(0), "deg_inv_sqrt length must equal num_nodes")


def spmm_gcn_forward_(row_ptr, col_ind, deg_inv_sqrt, x, out):
    """gcn_ops.cu:327 (naive) — same arithmetic as the plain kernel."""
    _gcn_checks(row_ptr, col_ind, deg_inv_sqrt, x, out)
    _spmm_call("gnn_spmm_gcn_forward", row_ptr, col_ind, deg_inv_sqrt, x, out)


def spmm_gcn_hmm_forward_(row_ptr, col_ind, deg_inv_sqrt, x, out):
    """gcn_ops.cu:350 ("plain", the default GCN aggregation)."""
    _gcn_checks(row_ptr, col_ind, deg_inv_sqrt, x, out)
    _spmm_call("gnn_spmm_gcn_hmm_forward", row_ptr, col_ind, deg_inv_sqrt, x, out)


def spmm_gcn_hmm_optimized_forward_(row_ptr, col_ind, deg_inv_sqrt, x, row_schedule, hot_feature_cache,
                                    hot_node_cutoff, out):
    """gcn_ops.cu:381 (row schedule + hot-row device cache)."""
    _gcn_checks(row_ptr, col_ind, deg_inv_sqrt, x, out)
    _check_optimized(row_schedule, hot_feature_cache, x, int(hot_node_cutoff))
    _spmm_call("gnn_spmm_gcn_hmm_optimized_forward", row_ptr, col_ind, deg_inv_sqrt, x, out,
               optimized=(row_schedule, hot_feature_cache, int(hot_node_cutoff)))


def stage_feature_pages_(page_ids, x, out, rows_per_page):
    """gcn_ops.cu:426 (checks :287-308)."""
    _check(page_ids.is_cuda, "page_ids must be CUDA")
    _check(out.is_cuda, "out must be CUDA")
    _check(page_ids.is_contiguous(), "page_ids must be contiguous")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(out.is_contiguous(), "out must be contiguous")
    _check(page_ids.dtype == torch.int64, "page_ids must be int64")
    _check(x.dtype == torch.float32, "x must be float32")
    _check(out.dtype == torch.float32, "out must be float32")
    _check(page_ids.dim() == 1, "page_ids must be rank-1")
    _check(x.dim() == 2, "x must be rank-2")
    _check(out.dim() == 2, "out must be rank-2")
    _check(int(rows_per_page) >= 1, "rows_per_page must be >= 1")
    _check(out.size(0) == page_ids.numel() * int(rows_per_page), "out rows must equal page_ids length * rows_per_page")
    _check(out.size(1) == x.size(1), "out feature dimension must match x")
    with torch.cuda.device(out.device):
        N.call("gnn_stage_feature_pages", _dev_ptr(page_ids), page_ids.numel(), _dev_ptr(x), x.size(0),
               _dev_ptr(out), int(rows_per_page), x.size(1), _stream(out.device))


def stage_feature_rows_(x, out):
    """gcn_ops.cu:449 (checks :310-323)."""
    _check(out.is_cuda, "out must be CUDA")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(out.is_contiguous(), "out must be contiguous")
    _check(x.dtype == torch.float32, "x must be float32")
    _check(out.dtype == torch.float32, "out must be float32")
    _check(x.dim() == 2, "x must be rank-2")
    _check(out.dim() == 2, "out must be rank-2")
    _check(out.size(0) <= x.size(0), "out rows must be <= x rows for staged prefix copies")
    _check(out.size(1) == x.size(1), "out feature dimension must match x")
    with torch.cuda.device(out.device):
        N.call("gnn_stage_feature_rows", _dev_ptr(x), x.size(0), _dev_ptr(out), out.size(0), x.size(1),
               _stream(out.device))


# ---------------------------------------------------------------------------
# pyg_gcn_ops table (pyg_gcn_ops.cpp:21-32)
# ---------------------------------------------------------------------------

def _pyg_checks(row_ptr, col_ind, edge_weight, x, out):
    _check_csr_common(row_ptr, col_ind, x, out, {"edge_weight": edge_weight})
    _check(col_ind.numel() == edge_weight.numel(), "col_ind and edge_weight lengths must match")


def spmm_pyg_gcn_forward_(row_ptr, col_ind, edge_weight, x, out):
    """pyg_gcn_ops.cu:254 (naive)."""
    _pyg_checks(row_ptr, col_ind, edge_weight, x, out)
    _spmm_call("gnn_spmm_pyg_gcn_forward", row_ptr, col_ind, edge_weight, x, out)


def spmm_pyg_gcn_plain_forward_(row_ptr, col_ind, edge_weight, x, out):
    """pyg_gcn_ops.cu:277 (plain)."""
    _pyg_checks(row_ptr, col_ind, edge_weight, x, out)
    _spmm_call("gnn_spmm_pyg_gcn_plain_forward", row_ptr, col_ind, edge_weight, x, out)


def _pyg_optimized(row_ptr, col_ind, edge_weight, x, row_schedule, hot_feature_cache, hot_node_cutoff, out):
    _pyg_checks(row_ptr, col_ind, edge_weight, x, out)
    _check_optimized(row_schedule, hot_feature_cache, x, int(hot_node_cutoff))
    _spmm_call("gnn_spmm_pyg_gcn_optimized_forward", row_ptr, col_ind, edge_weight, x, out,
               optimized=(row_schedule, hot_feature_cache, int(hot_node_cutoff)))


def spmm_pyg_gcn_hmm_optimized_forward_(row_ptr, col_ind, edge_weight, x, row_schedule, hot_feature_cache,
                                        hot_node_cutoff, out):
    """pyg_gcn_ops.cu:353."""
    _pyg_optimized(row_ptr, col_ind, edge_weight, x, row_schedule, hot_feature_cache, hot_node_cutoff, out)


def spmm_pyg_gcn_uvm_optimized_forward_(row_ptr, col_ind, edge_weight, x, row_schedule, hot_feature_cache,
                                        hot_node_cutoff, out):
    """pyg_gcn_ops.cu:363 (identical to the hmm entry in the reference)."""
    _pyg_optimized(row_ptr, col_ind, edge_weight, x, row_schedule, hot_feature_cache, hot_node_cutoff, out)


# ---------------------------------------------------------------------------
# agg_ops table (agg_ops.cpp:18-36)
# ---------------------------------------------------------------------------

def spmm_sum_forward_(row_ptr, col_ind, x, out):
    """agg_ops.cu:315."""
    _check_csr_common(row_ptr, col_ind, x, out, {})
    _spmm_call("gnn_spmm_sum_forward", row_ptr, col_ind, None, x, out)


def spmm_sum_hmm_forward_(row_ptr, col_ind, x, out):
    """agg_ops.cu:329 (same arithmetic as the plain sum)."""
    _check_csr_common(row_ptr, col_ind, x, out, {})
    _spmm_call("gnn_spmm_sum_forward", row_ptr, col_ind, None, x, out)


def spmm_mean_forward_(row_ptr, col_ind, x, out):
    """agg_ops.cu:322 — acc / deg."""
    _check_csr_common(row_ptr, col_ind, x, out, {})
    _spmm_call("gnn_spmm_mean_forward", row_ptr, col_ind, None, x, out, 0)


def spmm_mean_hmm_forward_(row_ptr, col_ind, x, out):
    """agg_ops.cu:336 — acc * (1 / deg)."""
    _check_csr_common(row_ptr, col_ind, x, out, {})
    _spmm_call("gnn_spmm_mean_forward", row_ptr, col_ind, None, x, out, 1)


def gemm_precision() -> int:
    """TF32 tensor cores when PyTorch allows TF32 matmuls (the reference's --tf32
    flag sets torch.backends.cuda.matmul.allow_tf32), full FP32 otherwise."""
    return N.GNN_PRECISION_TF32 if torch.backends.cuda.matmul.allow_tf32 else N.GNN_PRECISION_FP32


def _check_gemm(x, weight, out):
    """agg_ops.cu:263-280."""
    _check(out.is_cuda, "out must be CUDA")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(weight.is_contiguous(), "weight must be contiguous")
    _check(out.is_contiguous(), "out must be contiguous")
    _check(x.dtype == torch.float32, "x must be float32")
    _check(weight.dtype == torch.float32, "weight must be float32")
    _check(out.dtype == torch.float32, "out must be float32")
    _check(x.dim() == 2, "x must be rank-2")
    _check(weight.dim() == 2, "weight must be rank-2")
    _check(out.dim() == 2, "out must be rank-2")
    _check(x.size(1) == weight.size(0), "Inner GEMM dimensions must match")
    _check(out.size(0) == x.size(0) and out.size(1) == weight.size(1), "Output shape must match x @ weight")


def _check_bias(bias, out):
    if bias is not None and bias.numel() != 0:
        _check(bias.is_contiguous(), "bias must be contiguous")
        _check(bias.dtype == torch.float32, "bias must be float32")
        _check(bias.dim() == 1, "bias must be rank-1")
        _check(bias.numel() == out.size(1), "bias length must equal output feature dimension")


def gemm_forward_(x, weight, out, precision: int | None = None):
    """agg_ops.cu:369 — out = x @ weight."""
    _check_gemm(x, weight, out)
    p = gemm_precision() if precision is None else int(precision)
    with torch.cuda.device(out.device):
        N.call("gnn_gemm_forward", _dev_ptr(x), _dev_ptr(weight), out.data_ptr(), x.size(0), x.size(1),
               weight.size(1), p, _stream(out.device))


def linear_forward_(x, weight, bias, out, relu=False, precision: int | None = None):
    """agg_ops.cu:343 — out = relu?(x @ weight + bias), bias/ReLU fused into the GEMM epilogue."""
    _check_gemm(x, weight, out)
    _check_bias(bias, out)
    p = gemm_precision() if precision is None else int(precision)
    with torch.cuda.device(out.device):
        N.call("gnn_linear_forward", _dev_ptr(x), _dev_ptr(weight), _dev_ptr(bias), out.data_ptr(), x.size(0),
               x.size(1), weight.size(1), int(bool(relu)), p, _stream(out.device))


def linear_push_forward_(x, weight, bias, out, relu, peer_mask, peer_rows: list[int]) -> bool:
    """linear_forward_ (TF32 tensor-core path) that also stores every output row i to
    row i of peer_rows[d] (device addresses of the same [m, n] rows in peers' buffers)
    for each bit d of peer_mask[i] (uint8, one per row), from the GEMM's epilogue.
    Returns False, having launched nothing, where the tensor-core GEMM does not apply;
    the caller then runs linear_forward_ and a separate push."""
    _check_gemm(x, weight, out)
    _check_bias(bias, out)
    _check(peer_mask.is_cuda and peer_mask.dtype == torch.uint8 and peer_mask.is_contiguous(),
           "peer_mask must be a contiguous CUDA uint8 tensor")
    _check(peer_mask.numel() == out.size(0), "peer_mask needs one entry per output row")
    _check(len(peer_rows) <= 8, "at most 8 peers")
    if gemm_precision() != N.GNN_PRECISION_TF32:
        return False
    arr = (ctypes.c_void_p * max(1, len(peer_rows)))(*peer_rows)
    with torch.cuda.device(out.device):
        rc = N.lib().gnn_linear_push_forward(_dev_ptr(x), _dev_ptr(weight), _dev_ptr(bias), out.data_ptr(),
                                             x.size(0), x.size(1), weight.size(1), int(bool(relu)),
                                             peer_mask.data_ptr() if peer_mask.numel() else None, arr,
                                             len(peer_rows), _stream(out.device))
    if rc == N.GNN_ERR_UNSUPPORTED:
        return False
    N.check(rc, "gnn_linear_push_forward")
    return True


def bias_relu_forward_(out, bias, relu=False):
    """agg_ops.cu:393 (checks :282-295)."""
    _check(out.is_cuda, "out must be CUDA")
    _check(out.is_contiguous(), "out must be contiguous")
    _check(out.dtype == torch.float32, "out must be float32")
    _check(out.dim() == 2, "out must be rank-2")
    _check_bias(bias, out)
    with torch.cuda.device(out.device):
        N.call("gnn_bias_relu_forward", out.data_ptr(), _dev_ptr(bias), out.size(0), out.size(1),
               int(bool(relu)), _stream(out.device))


def tensor_add_inplace_(dst, src, alpha=1.0):
    """agg_ops.cu:399 — dst += alpha * src."""
    _check(dst.is_cuda, "dst must be CUDA")
    _check(dst.is_contiguous(), "dst must be contiguous")
    _check(src.is_contiguous(), "src must be contiguous")
    _check(dst.dtype == torch.float32, "dst must be float32")
    _check(src.dtype == torch.float32, "src must be float32")
    _check(tuple(dst.shape) == tuple(src.shape), "dst and src must have the same shape")
    with torch.cuda.device(dst.device):
        N.call("gnn_tensor_add_inplace", dst.data_ptr(), _dev_ptr(src), ctypes.c_float(float(alpha)),
               dst.numel(), _stream(dst.device))


def relu_inplace_(tensor):
    """agg_ops.cu:420."""
    _check(tensor.is_cuda, "tensor must be CUDA")
    _check(tensor.is_contiguous(), "tensor must be contiguous")
    _check(tensor.dtype == torch.float32, "tensor must be float32")
    with torch.cuda.device(tensor.device):
        N.call("gnn_relu_inplace", tensor.data_ptr(), tensor.numel(), _stream(tensor.device))


# ---------------------------------------------------------------------------
# uvm_allocator table (uvm_allocator.cpp:21-38)
# ---------------------------------------------------------------------------

_CODE_TO_DTYPE = {0: torch.float32, 1: torch.float64, 2: torch.float16, 3: torch.int32, 4: torch.int64}


class _ManagedBlock:
    """Owner of a cudaMallocManaged block exposed through __cuda_array_interface__.

    torch.as_tensor keeps a reference to this object; when the last tensor view
    dies the block is freed on its device (uvm_allocator.cu:107-113).
    """

    _TYPESTR = {torch.float32: "<f4", torch.float64: "<f8", torch.float16: "<f2", torch.int32: "<i4",
                torch.int64: "<i8", torch.uint8: "|u1"}

    def __init__(self, ptr: int, nbytes: int, shape, dtype: torch.dtype, device: int):
        self.ptr, self.nbytes, self.device = ptr, nbytes, device
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape),
            "typestr": self._TYPESTR[dtype],
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }

    def __del__(self):
        if self.ptr:
            try:
                N.lib().gnn_managed_free(ctypes.c_void_p(self.ptr), self.device)
            except Exception:
                pass
            self.ptr = 0


def managed_empty(sizes, dtype_code: int, device_index: int) -> torch.Tensor:
    """uvm_allocator.cu:93 — a CUDA tensor backed by cudaMallocManaged."""
    _check(int(device_index) >= 0, "device_index must be >= 0")
    _check(int(dtype_code) in _CODE_TO_DTYPE, f"Unsupported dtype code: {dtype_code}")
    dtype = _CODE_TO_DTYPE[int(dtype_code)]
    sizes = [int(s) for s in sizes]
    numel = 1
    for s in sizes:
        _check(s >= 0, f"Negative shape dimension: {s}")
        numel *= s
    nbytes = numel * torch.empty((), dtype=dtype).element_size()
    if nbytes == 0:
        return torch.empty(sizes, dtype=dtype, device=torch.device("cuda", int(device_index)))
    ptr = ctypes.c_void_p()
    N.check(N.lib().gnn_managed_alloc(nbytes, int(device_index), ctypes.byref(ptr)))
    block = _ManagedBlock(ptr.value, nbytes, sizes, dtype, int(device_index))
    with torch.cuda.device(int(device_index)):
        t = torch.as_tensor(block, device=torch.device("cuda", int(device_index)))
    _check(t.is_cuda, "Managed allocation did not materialize as a CUDA tensor")
    _check(t.data_ptr() == ptr.value, "Managed allocation was copied instead of wrapped")
    return t


def _hmm_supported(device_index: int) -> bool:
    v = ctypes.c_int(0)
    N.check(N.lib().gnn_hmm_supported(int(device_index), ctypes.byref(v)))
    return bool(v.value)


def hmm_empty(sizes, dtype_code: int, device_index: int) -> torch.Tensor:
    """uvm_allocator.cu:120 — an ordinary CPU tensor after an HMM capability check."""
    _check(int(device_index) >= 0, "device_index must be >= 0")
    _check(_hmm_supported(int(device_index)),
           "The selected CUDA device does not support Linux HMM pageable memory access")
    _check(int(dtype_code) in _CODE_TO_DTYPE, f"Unsupported dtype code: {dtype_code}")
    return torch.empty([int(s) for s in sizes], dtype=_CODE_TO_DTYPE[int(dtype_code)])


def copy_cpu_to_managed_(dst, src):
    """uvm_allocator.cu:129 — host memcpy into managed memory."""
    _check(dst.is_cuda, "Destination must be a CUDA managed tensor")
    _check(src.device.type == "cpu", "Source must be a CPU tensor")
    _check(dst.is_contiguous(), "Destination must be contiguous")
    _check(src.is_contiguous(), "Source must be contiguous")
    _check(dst.dtype == src.dtype, "Destination and source dtypes must match")
    _check(dst.numel() == src.numel(), "Destination and source shapes must have the same numel")
    nbytes = dst.numel() * dst.element_size()
    if nbytes == 0:
        return
    N.check(N.lib().gnn_copy_host_to_managed(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.data_ptr()), nbytes))


def _check_supported(t):
    _check(t.is_cuda or t.device.type == "cpu", "Expected a CPU or CUDA tensor")
    _check(t.is_contiguous(), "Expected a contiguous tensor")


def prefetch_(tensor, location_code: int, device_index: int, stream: int | None = None):
    """uvm_allocator.cu:151 — prefetch the whole tensor (on `stream`, default: current stream)."""
    prefetch_range_(tensor, 0, tensor.numel() * tensor.element_size(), location_code, device_index, stream)


def prefetch_range_(tensor, offset_bytes: int, byte_count: int, location_code: int, device_index: int,
                    stream: int | None = None):
    """uvm_allocator.cu:163."""
    _check_supported(tensor)
    _check(int(device_index) >= 0, "device_index must be >= 0")
    _check(int(offset_bytes) >= 0, "offset_bytes must be >= 0")
    _check(int(byte_count) >= 0, "byte_count must be >= 0")
    total = tensor.numel() * tensor.element_size()
    _check(int(offset_bytes) <= total, "offset_bytes exceeds tensor byte size")
    _check(int(byte_count) <= total - int(offset_bytes), "prefetch byte range exceeds tensor byte size")
    if int(byte_count) == 0:
        return
    if tensor.device.type == "cpu":
        _check(_hmm_supported(int(device_index)),
               "The selected CUDA device does not support Linux HMM pageable memory access")
    dev = torch.device("cuda", int(device_index))
    s = _stream(dev) if stream is None else int(stream)
    N.check(N.lib().gnn_prefetch(ctypes.c_void_p(tensor.data_ptr()), int(offset_bytes), int(byte_count), total,
                                 int(location_code), int(device_index), ctypes.c_void_p(s)))


def _advise(fn: str, tensor, location_code: int, device_index: int):
    _check_supported(tensor)
    if tensor.device.type == "cpu":
        _check(_hmm_supported(int(device_index)),
               "The selected CUDA device does not support Linux HMM pageable memory access")
    nbytes = tensor.numel() * tensor.element_size()
    N.check(getattr(N.lib(), fn)(ctypes.c_void_p(tensor.data_ptr()), nbytes, int(location_code), int(device_index)))


def advise_preferred_location_(tensor, location_code: int, device_index: int):
    """uvm_allocator.cu:189."""
    _advise("gnn_advise_preferred_location", tensor, location_code, device_index)


def advise_accessed_by_(tensor, location_code: int, device_index: int):
    """uvm_allocator.cu:202."""
    _advise("gnn_advise_accessed_by", tensor, location_code, device_index)


def advise_read_mostly_(tensor, enabled: bool):
    """uvm_allocator.cu:215."""
    _check_supported(tensor)
    device_index = tensor.get_device() if tensor.is_cuda else torch.cuda.current_device()
    if tensor.device.type == "cpu":
        _check(_hmm_supported(device_index),
               "The selected CUDA device does not support Linux HMM pageable memory access")
    nbytes = tensor.numel() * tensor.element_size()
    N.check(N.lib().gnn_advise_read_mostly(ctypes.c_void_p(tensor.data_ptr()), nbytes, int(bool(enabled)),
                                           int(device_index)))


def pointer_info(tensor) -> dict:
    """uvm_allocator.cu:231 — same keys and values as the reference's dict."""
    out = {
        "device_type": "cuda" if tensor.is_cuda else "cpu",
        "device_index": tensor.device.index if tensor.device.index is not None else -1,
        "is_managed": False,
        "is_host_mapped": False,
        "is_hmm": False,
        "pointer_type": "cpu" if tensor.device.type == "cpu" else "unknown",
    }
    if tensor.numel() == 0:
        return out
    info = N.gnn_pointer_info()
    N.check(N.lib().gnn_pointer_info_query(ctypes.c_void_p(tensor.data_ptr()), ctypes.byref(info)))
    if info.memory_type < 0:
        if tensor.device.type == "cpu" and info.pageable_access:
            out["is_hmm"] = True
            out["pointer_type"] = "hmm"
        return out
    out["is_managed"] = bool(info.is_managed)
    out["is_host_mapped"] = bool(info.is_host_mapped)
    is_hmm = tensor.device.type == "cpu" and not info.is_host_mapped and bool(info.pageable_access)
    out["is_hmm"] = is_hmm
    names = {0: "unregistered", 1: "host", 2: "device", 3: "managed"}
    out["pointer_type"] = ("host_mapped" if info.is_host_mapped else
                           ("hmm" if is_hmm else names.get(info.memory_type, "unknown")))
    return out


AGG_MODULE = SimpleNamespace(
    spmm_sum_forward_=spmm_sum_forward_, spmm_sum_hmm_forward_=spmm_sum_hmm_forward_,
    spmm_mean_forward_=spmm_mean_forward_, spmm_mean_hmm_forward_=spmm_mean_hmm_forward_,
    gemm_forward_=gemm_forward_, bias_relu_forward_=bias_relu_forward_, linear_forward_=linear_forward_,
    tensor_add_inplace_=tensor_add_inplace_, relu_inplace_=relu_inplace_)
GCN_MODULE = SimpleNamespace(
    spmm_gcn_forward_=spmm_gcn_forward_, spmm_gcn_hmm_forward_=spmm_gcn_hmm_forward_,
    spmm_gcn_hmm_optimized_forward_=spmm_gcn_hmm_optimized_forward_,
    stage_feature_pages_=stage_feature_pages_, stage_feature_rows_=stage_feature_rows_)
PYG_GCN_MODULE = SimpleNamespace(
    spmm_pyg_gcn_forward_=spmm_pyg_gcn_forward_, spmm_pyg_gcn_plain_forward_=spmm_pyg_gcn_plain_forward_,
    spmm_pyg_gcn_hmm_optimized_forward_=spmm_pyg_gcn_hmm_optimized_forward_,
    spmm_pyg_gcn_uvm_optimized_forward_=spmm_pyg_gcn_uvm_optimized_forward_)
ALLOCATOR_MODULE = SimpleNamespace(
    managed_empty=managed_empty, hmm_empty=hmm_empty, copy_cpu_to_managed_=copy_cpu_to_managed_,
    prefetch_=prefetch_, prefetch_range_=prefetch_range_, advise_preferred_location_=advise_preferred_location_,
    advise_accessed_by_=advise_accessed_by_, advise_read_mostly_=advise_read_mostly_, pointer_info=pointer_info)
