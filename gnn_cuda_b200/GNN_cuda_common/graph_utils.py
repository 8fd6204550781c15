"""CSR construction for the aggregation kernels (reference: GNN_cuda_common/graph_utils.py).

The CSR contract is the reference's and is reproduced bit for bit:
  * rows are destinations (incoming edges) unless ``transpose_for_incoming``
    is False; columns are sources;
  * self-loops are appended when asked (an existing loop merges with the new one);
  * duplicate (row, col) pairs collapse to one entry and columns are sorted
    within a row (scipy's ``tocsr()`` + ``sort_indices()`` in the reference);
  * ``deg_inv_sqrt = clip(deg, 1)^-0.5`` evaluated in float32 by numpy's power,
    and PyG edge weights ``dis[row] * dis[col]`` in float32;
  * ``row_ptr`` / ``col_ind`` are int32.
The construction here is a single sort of 64-bit (row, col) keys instead of a
sparse-matrix library conversion. Deviation, on purpose: where the reference's
int32 cast would silently wrap (more than 2^31-1 entries), ``index_dtype``
int32 raises, and ``index_dtype=torch.int64`` returns an int64 ``row_ptr``.

When ``src`` or ``dst`` is a CUDA tensor the CSR is built on that GPU by
libgnnb200 (``gnn_csr_build``: a radix sort of the keys, a unique pass and a
lower-bound search per row) and returned there; the same arrays bit for bit,
with ``deg_inv_sqrt`` looked up in a table of the same numpy float32 values.
CPU inputs keep the host construction, as in the reference.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch


@dataclass
class NormalizedCSR:
    row_ptr: torch.Tensor
    col_ind: torch.Tensor
    deg_inv_sqrt: torch.Tensor
    num_nodes: int
    num_edges: int


@dataclass
class PlainCSR:
    row_ptr: torch.Tensor
    col_ind: torch.Tensor
    num_nodes: int
    num_edges: int


@dataclass
class WeightedCSR:
    row_ptr: torch.Tensor
    col_ind: torch.Tensor
    edge_weight: torch.Tensor
    num_nodes: int
    num_edges: int


def default_gcn_preprocess_meta_path(dataset: str, *, data_root: str) -> str:
    return str(Path(data_root) / "gnn_cuda_preprocessed" / "gcn" / f"{dataset}.pt")


def feature_rows_per_page(*, feat_dim: int, page_bytes: int = 4096, dtype_bytes: int = 4) -> int:
    row_bytes = max(1, int(feat_dim) * int(dtype_bytes))
    return max(1, int(page_bytes) // row_bytes)


def apply_node_permutation(src, dst, features, *, perm, inv_perm):
    """Relabel nodes: new id of old node v is inv_perm[v]; feature row i of the
    result is old row perm[i]."""
    inv = torch.as_tensor(inv_perm).to(dtype=torch.long, device="cpu").contiguous()
    p = torch.as_tensor(perm).to(dtype=torch.long, device="cpu").contiguous()
    return inv[src.long().cpu()].contiguous(), inv[dst.long().cpu()].contiguous(), features[p].contiguous()


def apply_graph_permutation(src, dst, *, inv_perm):
    inv = torch.as_tensor(inv_perm).to(dtype=torch.long, device="cpu").contiguous()
    return inv[src.long().cpu()].contiguous(), inv[dst.long().cpu()].contiguous()


def _as_np(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().numpy().astype(np.int64, copy=False)
    return np.asarray(t, dtype=np.int64)


def csr_from_pairs(rows: np.ndarray, cols: np.ndarray, num_nodes: int) -> tuple[np.ndarray, np.ndarray]:
    """Sorted, de-duplicated CSR (int64 row_ptr, int64 col) of (row, col) pairs."""
    n = int(num_nodes)
    rows = np.asarray(rows, dtype=np.int64)
    cols = np.asarray(cols, dtype=np.int64)
    if rows.size:
        if rows.min() < 0:
            raise ValueError("negative row index found")
        if cols.min() < 0:
            raise ValueError("negative column index found")
        if rows.max() >= n:
            raise ValueError("row index exceeds matrix dimensions")
        if cols.max() >= n:
            raise ValueError("column index exceeds matrix dimensions")
    keys = np.unique(rows * np.int64(n) + cols) if rows.size else np.zeros(0, np.int64)
    r = keys // np.int64(max(n, 1))
    c = keys - r * np.int64(n)
    row_ptr = np.zeros(n + 1, dtype=np.int64)
    if n:
        np.cumsum(np.bincount(r, minlength=n), out=row_ptr[1:])
    return row_ptr, c


def _pairs(src, dst, num_nodes: int, add_self_loops: bool, dst_major: bool):
    s, d = _as_np(src), _as_np(dst)
    if add_self_loops:
        loop = np.arange(int(num_nodes), dtype=np.int64)
        s, d = np.concatenate([s, loop]), np.concatenate([d, loop])
    return (d, s) if dst_major else (s, d)


def _index(a: np.ndarray, dtype: torch.dtype, what: str) -> torch.Tensor:
    if dtype == torch.int32:
        if a.size and int(a.max()) > np.iinfo(np.int32).max:
            raise ValueError(f"{what} exceeds int32 range; pass index_dtype=torch.int64")
        return torch.from_numpy(a.astype(np.int32)).contiguous()
    return torch.from_numpy(a.astype(np.int64)).contiguous()


def deg_inv_sqrt_of(row_ptr: np.ndarray) -> np.ndarray:
    """float32 clip(deg, 1)^-0.5 through numpy's float32 power (the normalisation
    must be this exact float32 function to match the reference bit for bit)."""
    deg = np.diff(np.asarray(row_ptr, dtype=np.int64)).astype(np.float32)
    return np.power(np.clip(deg, np.float32(1.0), None), np.float32(-0.5)).astype(np.float32)


def _on_device(*ts) -> torch.device | None:
    for t in ts:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    return None


_DEVICE_ERRORS = ("negative row index found", "negative column index found", "row index exceeds matrix dimensions",
                  "column index exceeds matrix dimensions")


def device_csr(rows: torch.Tensor, cols: torch.Tensor, num_nodes: int, add_self_loops: bool,
               index_dtype: torch.dtype, device: torch.device) -> tuple[torch.Tensor, torch.Tensor, int]:
    """(row_ptr, col_ind, max_degree) of the (row, col) pairs, built on `device` by gnn_csr_build."""
    from .. import _native as N
    from . import native_ops
    if index_dtype not in (torch.int32, torch.int64):
        raise ValueError("index_dtype must be torch.int32 or torch.int64")
    r = torch.as_tensor(rows).to(device=device, dtype=torch.int64).contiguous()
    c = torch.as_tensor(cols).to(device=device, dtype=torch.int64).contiguous()
    if r.numel() != c.numel():
        raise ValueError("row and column arrays must have the same length")
    n, e, loops = int(num_nodes), int(r.numel()), int(bool(add_self_loops))
    L = N.lib()
    with torch.cuda.device(device):
        wsb = int(L.gnn_csr_build_workspace_bytes(e, n, loops))
        if wsb == 0:
            raise RuntimeError(N.last_error() or "gnn_csr_build_workspace_bytes failed")
        ws = torch.empty(wsb, dtype=torch.uint8, device=device)
        cap = e + (n if loops else 0)
        row_ptr = torch.empty(n + 1, dtype=index_dtype, device=device)
        col = torch.empty(max(cap, 1), dtype=torch.int32, device=device)
        nu, md = ctypes.c_int64(0), ctypes.c_int64(0)
        idx = N.GNN_INDEX_INT64 if index_dtype == torch.int64 else N.GNN_INDEX_INT32
        status = L.gnn_csr_build(r.data_ptr(), c.data_ptr(), e, n, loops, row_ptr.data_ptr(), idx, col.data_ptr(), cap,
                                 ctypes.byref(nu), ctypes.byref(md), ws.data_ptr(), wsb, native_ops._stream(device))
        if status != N.GNN_OK:
            msg = N.last_error()
            if msg in _DEVICE_ERRORS:
                raise ValueError(msg)
            if msg.startswith("row_ptr exceeds int32 range"):
                raise ValueError("row_ptr exceeds int32 range; pass index_dtype=torch.int64")
            N.check(status, "gnn_csr_build")
    return row_ptr, col[:nu.value], int(md.value)


def device_deg_inv_sqrt(row_ptr: torch.Tensor, num_nodes: int, max_degree: int) -> torch.Tensor:
    """deg_inv_sqrt on row_ptr's device from a host table of numpy's float32 clip(d, 1)^-0.5."""
    from .. import _native as N
    from . import native_ops
    dev = row_ptr.device
    table = np.power(np.clip(np.arange(max(int(max_degree), 1) + 1).astype(np.float32), np.float32(1.0), None),
                     np.float32(-0.5)).astype(np.float32)
    t_table = torch.from_numpy(table).to(dev)
    dis = torch.empty(int(num_nodes), dtype=torch.float32, device=dev)
    idx = N.GNN_INDEX_INT64 if row_ptr.dtype == torch.int64 else N.GNN_INDEX_INT32
    with torch.cuda.device(dev):
        N.call("gnn_csr_deg_inv_sqrt", row_ptr.data_ptr(), idx, int(num_nodes), t_table.data_ptr(), table.shape[0],
               dis.data_ptr(), native_ops._stream(dev))
    return dis


def device_edge_weight(row_ptr: torch.Tensor, col_ind: torch.Tensor, dis: torch.Tensor) -> torch.Tensor:
    from .. import _native as N
    from . import native_ops
    dev = row_ptr.device
    ew = torch.empty(int(col_ind.numel()), dtype=torch.float32, device=dev)
    idx = N.GNN_INDEX_INT64 if row_ptr.dtype == torch.int64 else N.GNN_INDEX_INT32
    with torch.cuda.device(dev):
        N.call("gnn_csr_edge_weight", row_ptr.data_ptr(), idx, col_ind.data_ptr(), dis.data_ptr(), int(dis.numel()),
               ew.data_ptr(), native_ops._stream(dev))
    return ew


def build_gcn_normalized_csr(src, dst, *, num_nodes: int, add_self_loops: bool = True,
                             index_dtype: torch.dtype = torch.int32) -> NormalizedCSR:
    dev = _on_device(src, dst)
    if dev is not None:
        row_ptr, col, md = device_csr(dst, src, num_nodes, add_self_loops, index_dtype, dev)
        return NormalizedCSR(row_ptr=row_ptr, col_ind=col, deg_inv_sqrt=device_deg_inv_sqrt(row_ptr, num_nodes, md),
                             num_nodes=int(num_nodes), num_edges=int(col.numel()))
    r, c = _pairs(src, dst, num_nodes, add_self_loops, dst_major=True)
    row_ptr, col = csr_from_pairs(r, c, num_nodes)
    return NormalizedCSR(row_ptr=_index(row_ptr, index_dtype, "row_ptr"), col_ind=_index(col, torch.int32, "col_ind"),
                         deg_inv_sqrt=torch.from_numpy(deg_inv_sqrt_of(row_ptr)).contiguous(),
                         num_nodes=int(num_nodes), num_edges=int(col.shape[0]))


def build_pyg_gcn_weighted_csr(src, dst, *, num_nodes: int, add_self_loops: bool = True,
                               index_dtype: torch.dtype = torch.int32) -> WeightedCSR:
    dev = _on_device(src, dst)
    if dev is not None:
        row_ptr, col, md = device_csr(dst, src, num_nodes, add_self_loops, index_dtype, dev)
        dis = device_deg_inv_sqrt(row_ptr, num_nodes, md)
        return WeightedCSR(row_ptr=row_ptr, col_ind=col, edge_weight=device_edge_weight(row_ptr, col, dis),
                           num_nodes=int(num_nodes), num_edges=int(col.numel()))
    r, c = _pairs(src, dst, num_nodes, add_self_loops, dst_major=True)
    row_ptr, col = csr_from_pairs(r, c, num_nodes)
    dis = deg_inv_sqrt_of(row_ptr)
    row_of_edge = np.repeat(np.arange(int(num_nodes), dtype=np.int64), np.diff(row_ptr))
    ew = (dis[row_of_edge] * dis[col]).astype(np.float32)
    return WeightedCSR(row_ptr=_index(row_ptr, index_dtype, "row_ptr"), col_ind=_index(col, torch.int32, "col_ind"),
                       edge_weight=torch.from_numpy(ew).contiguous(), num_nodes=int(num_nodes),
                       num_edges=int(col.shape[0]))


def build_plain_csr(src, dst, *, num_nodes: int, add_self_loops: bool = False, transpose_for_incoming: bool = True,
                    index_dtype: torch.dtype = torch.int32) -> PlainCSR:
    dev = _on_device(src, dst)
    if dev is not None:
        rows, cols = (dst, src) if transpose_for_incoming else (src, dst)
        row_ptr, col, _ = device_csr(rows, cols, num_nodes, add_self_loops, index_dtype, dev)
        return PlainCSR(row_ptr=row_ptr, col_ind=col, num_nodes=int(num_nodes), num_edges=int(col.numel()))
    r, c = _pairs(src, dst, num_nodes, add_self_loops, dst_major=transpose_for_incoming)
    row_ptr, col = csr_from_pairs(r, c, num_nodes)
    return PlainCSR(row_ptr=_index(row_ptr, index_dtype, "row_ptr"), col_ind=_index(col, torch.int32, "col_ind"),
                    num_nodes=int(num_nodes), num_edges=int(col.shape[0]))


def load_src_dst_features(loaded, *, load_kind: str):
    if load_kind == "pyg":
        edge_index, features, num_nodes = loaded
        return edge_index[0].contiguous(), edge_index[1].contiguous(), features, num_nodes
    if load_kind == "dgl":
        src, dst, features, num_nodes = loaded
        return src.contiguous(), dst.contiguous(), features, num_nodes
    raise ValueError(f"Unsupported load_kind: {load_kind}")


def resolve_dataset_path(dataset: str, *, data_root: str) -> str:
    if dataset == "all":
        raise ValueError("'all' is only supported by the run/ entrypoints")
    if "/" in dataset or "\\" in dataset or dataset.endswith(".npz"):
        raise ValueError("--dataset only accepts a dataset name or 'all'")
    return str(Path(data_root) / f"{dataset}.npz")


# UVM locality preprocessing (graph_utils.py:174-446 of the reference), computed on the GPU.
from .locality import (  # noqa: E402,F401  (re-exported under the reference's module)
    build_coaccess_feature_permutation,
    build_hot_partition_feature_permutation,
    build_page_reuse_schedule_metadata,
)
