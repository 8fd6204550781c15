"""UVM locality preprocessing on the GPU (reference: GNN_cuda_common/graph_utils.py:174-446
and run/preprocess_gcn_graph.py:40-146).

The reference computes, on the host with per-row / per-window Python loops,
the metadata that ``--spmm_mode optimized`` consumes: a row schedule that
groups rows reading the same feature pages, per-block and per-window hot page
lists, a co-access node order, and a hot-prefix/cold-suffix node permutation.
The functions here keep the reference's names, keyword arguments, defaults and
return values (dicts with the same keys, ``(perm, inv_perm)`` tuples), and run
every step on a GPU through libgnnb200 (``gnn_locality_*``): the same arrays
bit for bit, the same float64 ratios.

Placement: the computation always runs on a CUDA device (the inputs' device
when they are CUDA tensors, else the current device). Results come back where
the inputs were: CPU tensors for CPU inputs, as the reference returns, device
tensors for device inputs. There is no CPU fallback: without a CUDA device these
functions raise.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _native as N
from . import native_ops


def device_csr(*args, **kwargs):
    # graph_utils re-exports this module's functions, so it is imported on use, not at import time
    from .graph_utils import device_csr as build
    return build(*args, **kwargs)


def feature_rows_per_page(**kwargs) -> int:
    from .graph_utils import feature_rows_per_page as rows
    return rows(**kwargs)


def _compute_device(*ts) -> torch.device:
    for t in ts:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("locality preprocessing runs on a CUDA device and none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _result_device(*ts) -> torch.device:
    for t in ts:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    return torch.device("cpu")


def _ids(t, dev: torch.device) -> torch.Tensor:
    return torch.as_tensor(t).to(device=dev, dtype=torch.int64).contiguous()


def _workspace(dev: torch.device, n: int, e: int, k: int) -> torch.Tensor:
    nbytes = int(N.lib().gnn_locality_workspace_bytes(int(n), int(e), int(k)))
    if nbytes == 0:
        raise RuntimeError(N.last_error() or "gnn_locality_workspace_bytes failed")
    return torch.empty(nbytes, dtype=torch.uint8, device=dev)


def _csr(src, dst, num_nodes: int, add_self_loops: bool, dev: torch.device):
    # graph_utils.py:258-267: dst-major CSR of (dst, src) (+ loops), merged duplicates, sorted columns
    row_ptr, col, _ = device_csr(dst, src, num_nodes, add_self_loops, torch.int64, dev)
    return row_ptr, col


def page_schedule_from_csr(row_ptr: torch.Tensor, col_ind: torch.Tensor, *, num_nodes: int, rows_per_page: int,
                           row_block_size: int = 64, hot_cache_pages: int = 1024, signature_topk: int = 4,
                           window_num_blocks: int = 4, window_cache_pages: int = 8) -> dict:
    """Page metadata of a device CSR; device tensors under the reference's keys."""
    dev = row_ptr.device
    n, e = int(num_nodes), int(col_ind.numel())
    rpp = int(rows_per_page)
    rbs = int(row_block_size)
    if rbs < 1:
        raise ValueError("row_block_size must be >= 1")
    k = max(1, int(signature_topk))
    wnb = max(1, int(window_num_blocks))
    wcp = max(1, int(window_cache_pages))
    rpw = rbs * wnb
    num_pages = (n + rpp - 1) // rpp
    nb = (n + rbs - 1) // rbs
    nw = (n + rpw - 1) // rpw
    hcp = max(0, min(int(hot_cache_pages), num_pages))
    page_hist = torch.empty(num_pages, dtype=torch.int64, device=dev)
    hot_pages = torch.empty(hcp, dtype=torch.int64, device=dev)
    schedule = torch.empty(n, dtype=torch.int64, device=dev)
    block_hot = torch.empty(nb, k, dtype=torch.int64, device=dev)
    window_hot = torch.empty(nw, wcp, dtype=torch.int64, device=dev)
    maxc = ctypes.c_int64(0)
    hot_cov, win_cov = ctypes.c_double(0.0), ctypes.c_double(0.0)
    idx = N.GNN_INDEX_INT64 if row_ptr.dtype == torch.int64 else N.GNN_INDEX_INT32
    with torch.cuda.device(dev):
        ws = _workspace(dev, n, e, max(k, wcp))
        N.call("gnn_locality_page_schedule", row_ptr.data_ptr(), idx, col_ind.data_ptr() if e else None, n, e, rpp,
               rbs, wnb, wcp, hcp, k, page_hist.data_ptr(), hot_pages.data_ptr() if hcp else None,
               schedule.data_ptr(), block_hot.data_ptr(), window_hot.data_ptr(), ctypes.byref(maxc),
               ctypes.byref(hot_cov), ctypes.byref(win_cov), ws.data_ptr(), ws.numel(), native_ops._stream(dev))
        reuse = torch.empty(int(maxc.value) + 1, dtype=torch.int64, device=dev)
        N.call("gnn_locality_count_histogram", page_hist.data_ptr(), num_pages, reuse.data_ptr(), reuse.numel(),
               native_ops._stream(dev))
    return {
        "rows_per_page": rpp, "num_pages": num_pages, "page_histogram": page_hist, "page_reuse_histogram": reuse,
        "hot_pages": hot_pages, "hot_coverage": float(hot_cov.value), "row_schedule": schedule,
        "row_block_size": rbs, "block_hot_pages": block_hot, "window_num_blocks": wnb, "window_cache_pages": wcp,
        "rows_per_window": rpw, "window_hot_pages": window_hot, "avg_window_hot_coverage": float(win_cov.value),
        "signature_topk": k,
    }


def _to(meta: dict, dev: torch.device) -> dict:
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in meta.items()}


def build_page_reuse_schedule_metadata(src, dst, *, num_nodes: int, feat_dim: int, page_bytes: int = 4096,
                                       row_block_size: int = 64, hot_cache_pages: int = 1024,
                                       signature_topk: int = 4, window_num_blocks: int = 4,
                                       window_cache_pages: int = 8, add_self_loops: bool = True) -> dict:
    """graph_utils.py:244-372 on the GPU: page histogram and reuse histogram,
    hot pages and their coverage, the row schedule (rows sorted by their top-k
    page signature, then degree descending), and the top pages of every
    row block and row window of that schedule."""
    dev = _compute_device(src, dst)
    row_ptr, col = _csr(src, dst, num_nodes, add_self_loops, dev)
    meta = page_schedule_from_csr(row_ptr, col, num_nodes=num_nodes,
                                  rows_per_page=feature_rows_per_page(feat_dim=int(feat_dim), page_bytes=int(page_bytes)),
                                  row_block_size=row_block_size, hot_cache_pages=hot_cache_pages,
                                  signature_topk=signature_topk, window_num_blocks=window_num_blocks,
                                  window_cache_pages=window_cache_pages)
    meta["page_bytes"] = int(page_bytes)
    return _to(meta, _result_device(src, dst))


def coaccess_from_csr(row_ptr: torch.Tensor, col_ind: torch.Tensor, *, num_nodes: int, row_schedule: torch.Tensor,
                      rows_per_window: int, signature_topk: int = 4) -> tuple[torch.Tensor, torch.Tensor]:
    dev = row_ptr.device
    n, e = int(num_nodes), int(col_ind.numel())
    sched = _ids(row_schedule, dev)
    if int(sched.numel()) != n:
        raise ValueError("row_schedule must contain exactly num_nodes entries")
    k = max(1, int(signature_topk))
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    inv = torch.empty(n, dtype=torch.int64, device=dev)
    idx = N.GNN_INDEX_INT64 if row_ptr.dtype == torch.int64 else N.GNN_INDEX_INT32
    with torch.cuda.device(dev):
        ws = _workspace(dev, n, e, k)
        N.call("gnn_locality_coaccess_permutation", row_ptr.data_ptr(), idx, col_ind.data_ptr() if e else None, n, e,
               sched.data_ptr(), max(1, int(rows_per_window)), k, perm.data_ptr(), inv.data_ptr(), ws.data_ptr(),
               ws.numel(), native_ops._stream(dev))
    return perm, inv


def build_coaccess_feature_permutation(src, dst, *, num_nodes: int, row_schedule, row_block_size: int = 64,
                                       window_num_blocks: int = 4, signature_topk: int = 4,
                                       add_self_loops: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """graph_utils.py:375-446 on the GPU: nodes ordered by the row-schedule
    windows that read them most (top-k windows by read count, ties to the
    earlier window), then by total reads descending, then by id."""
    dev = _compute_device(src, dst, row_schedule)
    row_ptr, col = _csr(src, dst, num_nodes, add_self_loops, dev)
    perm, inv = coaccess_from_csr(row_ptr, col, num_nodes=num_nodes, row_schedule=row_schedule,
                                  rows_per_window=max(1, int(row_block_size) * int(window_num_blocks)),
                                  signature_topk=signature_topk)
    out = _result_device(src, dst)
    return perm.to(out), inv.to(out)


def build_hot_partition_feature_permutation(src, *, num_nodes: int, base_order=None,
                                            hot_access_coverage: float = 0.80, hot_max_ratio: float = 0.25,
                                            hot_min_nodes: int = 256, add_self_loops: bool = True) -> dict:
    """graph_utils.py:174-241 on the GPU: the most-read nodes (enough to cover
    `hot_access_coverage` of all reads, clamped to [hot_min_nodes,
    ceil(hot_max_ratio * num_nodes)]) moved to the front of `base_order` (or
    all nodes by reads descending when there is none)."""
    dev = _compute_device(src, base_order)
    n = int(num_nodes)
    s = _ids(src, dev)
    base = None
    if base_order is not None:
        base = _ids(base_order, dev)
        if int(base.numel()) != n:
            raise ValueError("base_order must contain exactly num_nodes entries")
    access = torch.empty(n, dtype=torch.int64, device=dev)
    order = torch.empty(n, dtype=torch.int64, device=dev)
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    inv = torch.empty(n, dtype=torch.int64, device=dev)
    cutoff, min_used, total, hot = (ctypes.c_int64(0) for _ in range(4))
    with torch.cuda.device(dev):
        ws = _workspace(dev, n, 0, 1)
        N.call("gnn_locality_hot_partition", s.data_ptr() if s.numel() else None, int(s.numel()), n,
               int(bool(add_self_loops)), base.data_ptr() if base is not None else None, float(hot_access_coverage),
               float(hot_max_ratio), int(hot_min_nodes), access.data_ptr(), order.data_ptr(), perm.data_ptr(),
               inv.data_ptr(), ctypes.byref(cutoff), ctypes.byref(min_used), ctypes.byref(total), ctypes.byref(hot),
               ws.data_ptr(), ws.numel(), native_ops._stream(dev))
    c, t, h = int(cutoff.value), int(total.value), int(hot.value)
    out = _result_device(src, base_order)
    cov = float(max(0.0, min(1.0, float(hot_access_coverage))))
    return {
        "perm": perm.to(out), "inv_perm": inv.to(out), "hot_nodes": order[:c].contiguous().to(out),
        "hot_node_cutoff": c, "hot_node_fraction": float(c / max(1, n)),
        "hot_node_access_coverage": float(h / t) if t > 0 else 0.0,
        "hot_node_access_counts": access.to(out), "hot_total_accesses": t, "hot_access_target": cov,
        "hot_max_ratio": float(hot_max_ratio), "hot_min_nodes": int(min_used.value),
    }


def apply_graph_permutation_device(src: torch.Tensor, dst: torch.Tensor, *, inv_perm: torch.Tensor):
    """apply_graph_permutation (graph_utils.py:76-85) for CUDA tensors, on their device."""
    dev = _compute_device(src, dst, inv_perm)
    s, d, inv = _ids(src, dev), _ids(dst, dev), _ids(inv_perm, dev)
    if s.numel() != d.numel():
        raise ValueError("src and dst must have the same length")
    so, do = torch.empty_like(s), torch.empty_like(d)
    with torch.cuda.device(dev):
        flag = torch.empty(256, dtype=torch.uint8, device=dev)
        N.call("gnn_permute_edges", s.data_ptr() if s.numel() else None, d.data_ptr() if d.numel() else None,
               int(s.numel()), inv.data_ptr(), int(inv.numel()), so.data_ptr() if s.numel() else None,
               do.data_ptr() if d.numel() else None, flag.data_ptr(), 256, native_ops._stream(dev))
    return so, do


def preprocess_gcn_graph(src, dst, *, num_nodes: int, feat_dim: int = 128, page_bytes: int = 4096,
                         row_block_size: int = 64, window_num_blocks: int = 4, window_cache_pages: int = 8,
                         hot_cache_pages: int = 1024, signature_topk: int = 4, hot_access_coverage: float = 0.80,
                         hot_max_ratio: float = 0.25, hot_min_nodes: int = 256) -> dict:
    """The whole chain of run/preprocess_gcn_graph.py:40-120 on one GPU: page
    schedule of the graph -> co-access order -> hot partition of that order ->
    renumbered graph -> its page schedule. Returns the saved payload's fields
    (perm/inv_perm/hot_* of the partition and the final page metadata), with
    tensors on the inputs' device (CPU for CPU inputs)."""
    dev = _compute_device(src, dst)
    out = _result_device(src, dst)
    s, d = _ids(src, dev), _ids(dst, dev)
    n = int(num_nodes)
    rpp = feature_rows_per_page(feat_dim=int(feat_dim), page_bytes=int(page_bytes))
    page_kw = dict(rows_per_page=rpp, row_block_size=row_block_size, hot_cache_pages=hot_cache_pages,
                   signature_topk=signature_topk, window_num_blocks=window_num_blocks,
                   window_cache_pages=window_cache_pages)
    rp, col = _csr(s, d, n, True, dev)
    base = page_schedule_from_csr(rp, col, num_nodes=n, **page_kw)
    perm, _ = coaccess_from_csr(rp, col, num_nodes=n, row_schedule=base["row_schedule"],
                                rows_per_window=max(1, int(row_block_size) * max(1, int(window_num_blocks))),
                                signature_topk=signature_topk)
    del rp, col, base
    hot = build_hot_partition_feature_permutation(s, num_nodes=n, base_order=perm,
                                                  hot_access_coverage=hot_access_coverage,
                                                  hot_max_ratio=hot_max_ratio, hot_min_nodes=hot_min_nodes,
                                                  add_self_loops=True)
    s_r, d_r = apply_graph_permutation_device(s, d, inv_perm=hot["inv_perm"])
    rp, col = _csr(s_r, d_r, n, True, dev)
    final = page_schedule_from_csr(rp, col, num_nodes=n, **page_kw)
    final["page_bytes"] = int(page_bytes)
    payload = {
        "num_nodes": n, "feat_dim": int(feat_dim), "strategy": "hot_node_partition+coaccess_feature_reorder",
        "add_self_loops": True, "perm": hot["perm"], "inv_perm": hot["inv_perm"], "hot_nodes": hot["hot_nodes"],
        "hot_node_cutoff": hot["hot_node_cutoff"], "hot_node_fraction": hot["hot_node_fraction"],
        "hot_node_access_coverage": hot["hot_node_access_coverage"],
        "hot_node_access_counts": hot["hot_node_access_counts"], "hot_total_accesses": hot["hot_total_accesses"],
        "hot_access_target": hot["hot_access_target"], "hot_max_ratio": hot["hot_max_ratio"],
        "hot_min_nodes": hot["hot_min_nodes"], **final,
    }
    return _to(payload, out)


__all__ = [
    "build_page_reuse_schedule_metadata", "build_coaccess_feature_permutation",
    "build_hot_partition_feature_permutation", "apply_graph_permutation_device", "preprocess_gcn_graph",
    "page_schedule_from_csr", "coaccess_from_csr",
]
