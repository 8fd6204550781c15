"""CPU oracle for the UVM locality preprocessing (row schedule, page metadata,
co-access order, hot-prefix partition).

TEST INFRASTRUCTURE ONLY — the test oracle, never the product. Only ``tests/``
import this module; nothing under ``gnn_cuda_b200/`` may import it.

A vectorised numpy restatement of the reference's host implementation,
function by function:
  * ``page_reuse_schedule``  — graph_utils.py:244-372 (build_page_reuse_schedule_metadata)
  * ``coaccess_permutation`` — graph_utils.py:375-446 (build_coaccess_feature_permutation)
  * ``hot_partition``        — graph_utils.py:174-241 (build_hot_partition_feature_permutation)
  * ``preprocess``           — the chain of run/preprocess_gcn_graph.py:40-120
The reference walks rows, blocks and windows in Python loops with per-row
``np.unique``/``np.lexsort``; here the same orders come from whole-array
sorts: a "top-k per segment" is a lexsort of the distinct (segment, item)
pairs by (segment, count descending, tie key) followed by the first k of every
segment. Pinned bit for bit against ``tests/golden/locality_cases.npz``, which
``tests/golden/make_locality_golden.py`` produced by running the reference's
own functions.
"""
from __future__ import annotations

import numpy as np

from .oracle import _coo_to_csr, _with_loops


def rows_per_page(feat_dim: int, page_bytes: int = 4096, dtype_bytes: int = 4) -> int:
    """graph_utils.py:43-50: feature rows that fit one host page (at least 1)."""
    return max(1, int(page_bytes) // max(1, int(feat_dim) * int(dtype_bytes)))


def _csr(src, dst, num_nodes: int, add_self_loops: bool):
    # graph_utils.py:258-267: dst-major CSR of (dst, src) + loops, duplicates merged, columns sorted
    s, d = _with_loops(src, dst, num_nodes, add_self_loops)
    csr = _coo_to_csr(d, s, num_nodes)
    return csr.indptr.astype(np.int64), csr.indices.astype(np.int64)


def _stable_desc(values: np.ndarray) -> np.ndarray:
    """Indices ordering `values` largest first, equal values in index order."""
    return np.argsort(-values.astype(np.int64), kind="stable")


def _segment_topk(seg: np.ndarray, item: np.ndarray, num_segments: int, num_items: int, k: int,
                  tie: np.ndarray | None = None):
    """For every segment, the k distinct items occurring most often in it, ties
    by the smaller `tie[item]` (item itself when tie is None).
    Returns (items [S, k] padded with num_items, counts [S, k] padded with 0,
    per-segment total count [S])."""
    key = seg.astype(np.int64) * np.int64(num_items) + item.astype(np.int64)
    ukey, cnt = np.unique(key, return_counts=True)
    useg = ukey // num_items
    uitem = ukey % num_items
    tkey = uitem if tie is None else tie[uitem]
    order = np.lexsort((tkey, -cnt, useg))
    useg, uitem, cnt = useg[order], uitem[order], cnt[order]
    first = np.searchsorted(useg, np.arange(num_segments, dtype=np.int64), side="left")
    pos = np.arange(useg.size, dtype=np.int64) - first[useg] if useg.size else np.zeros(0, np.int64)
    keep = pos < k
    items = np.full((num_segments, k), num_items, dtype=np.int64)
    counts = np.zeros((num_segments, k), dtype=np.int64)
    items[useg[keep], pos[keep]] = uitem[keep]
    counts[useg[keep], pos[keep]] = cnt[keep]
    total = np.zeros(num_segments, dtype=np.int64)
    np.add.at(total, useg, cnt)
    return items, counts, total


def _lexsort_rows(num: int, keys_minor_to_major: list[np.ndarray]) -> np.ndarray:
    """np.lexsort with the identity as the least significant key."""
    return np.lexsort(tuple([np.arange(num, dtype=np.int64), *keys_minor_to_major])).astype(np.int64)


def page_reuse_schedule(src, dst, *, num_nodes: int, feat_dim: int, page_bytes: int = 4096,
                        row_block_size: int = 64, hot_cache_pages: int = 1024, signature_topk: int = 4,
                        window_num_blocks: int = 4, window_cache_pages: int = 8, add_self_loops: bool = True) -> dict:
    """graph_utils.py:244-372. Returns numpy arrays / Python scalars under the reference's keys."""
    n = int(num_nodes)
    row_ptr, col = _csr(src, dst, n, add_self_loops)
    rpp = rows_per_page(feat_dim, page_bytes)
    num_pages = (n + rpp - 1) // rpp
    page = col // rpp
    page_hist = np.bincount(page, minlength=num_pages).astype(np.int64)
    nz = page_hist[page_hist > 0]
    reuse = np.bincount(nz).astype(np.int64) if nz.size else np.zeros(1, np.int64)
    degree = np.diff(row_ptr)
    hot_order = _stable_desc(page_hist)
    hcp = max(0, min(int(hot_cache_pages), num_pages))
    hot_pages = hot_order[:hcp].astype(np.int64)
    total = int(page_hist.sum())
    hot_cov = float(page_hist[hot_pages].sum() / total) if hot_pages.size > 0 and total > 0 else 0.0
    rank = np.empty(num_pages, np.int64)
    rank[hot_order] = np.arange(num_pages, dtype=np.int64)
    k = max(1, int(signature_topk))
    rows = np.repeat(np.arange(n, dtype=np.int64), degree)
    # row signature: the row's k pages by (entries desc, page rank asc), padded with num_pages (:297-306)
    sig, _, _ = _segment_topk(rows, page, n, num_pages, k, tie=rank)
    keys = [-degree] + [sig[:, j] for j in range(k - 1, -1, -1)]
    row_schedule = _lexsort_rows(n, keys)  # (:308-311)
    slot = np.empty(n, np.int64)
    slot[row_schedule] = np.arange(n, dtype=np.int64)
    rbs = int(row_block_size)
    num_blocks = (n + rbs - 1) // rbs
    block_hot, _, _ = _segment_topk(slot[rows] // rbs, page, num_blocks, num_pages, k, tie=rank)  # (:313-334)
    wnb = max(1, int(window_num_blocks))
    wcp = max(1, int(window_cache_pages))
    rpw = rbs * wnb
    num_windows = (n + rpw - 1) // rpw
    win_hot, win_cnt, win_total = _segment_topk(slot[rows] // rpw, page, num_windows, num_pages, wcp, tie=rank)
    # per-window covered fraction, summed window by window in float64 (:336-356)
    covered = win_cnt.sum(axis=1)
    ratio = np.where(win_total > 0, covered / np.maximum(win_total, 1), 0.0).astype(np.float64)
    cov_sum = float(np.add.accumulate(ratio)[-1]) if ratio.size else 0.0
    return {
        "rows_per_page": rpp, "num_pages": num_pages, "page_histogram": page_hist, "page_reuse_histogram": reuse,
        "hot_pages": hot_pages, "hot_coverage": hot_cov, "row_schedule": row_schedule, "row_block_size": rbs,
        "block_hot_pages": block_hot, "window_num_blocks": wnb, "window_cache_pages": wcp, "rows_per_window": rpw,
        "window_hot_pages": win_hot, "avg_window_hot_coverage": float(cov_sum / max(1, num_windows)),
        "signature_topk": k, "page_bytes": int(page_bytes),
    }


def coaccess_permutation(src, dst, *, num_nodes: int, row_schedule: np.ndarray, row_block_size: int = 64,
                         window_num_blocks: int = 4, signature_topk: int = 4, add_self_loops: bool = True):
    """graph_utils.py:375-446: nodes ordered by the windows (of the row schedule)
    that read them most. Returns (perm, inv_perm) int64."""
    n = int(num_nodes)
    row_ptr, col = _csr(src, dst, n, add_self_loops)
    rpw = max(1, int(row_block_size) * int(window_num_blocks))
    num_windows = (n + rpw - 1) // rpw
    k = max(1, int(signature_topk))
    slot = np.empty(n, np.int64)
    slot[np.asarray(row_schedule, dtype=np.int64)] = np.arange(n, dtype=np.int64)
    rows = np.repeat(np.arange(n, dtype=np.int64), np.diff(row_ptr))
    access = np.bincount(col, minlength=n).astype(np.int64)
    # per node: the k windows reading it most, ties by smaller window (:418-425)
    top_w, top_c, _ = _segment_topk(col, slot[rows] // rpw, n, num_windows, k)
    keys = [-access]
    for j in range(k - 1, -1, -1):
        keys += [-top_c[:, j], top_w[:, j]]
    perm = _lexsort_rows(n, keys)  # (:427-432)
    inv = np.empty(n, np.int64)
    inv[perm] = np.arange(n, dtype=np.int64)
    return perm, inv


def hot_partition(src, *, num_nodes: int, base_order=None, hot_access_coverage: float = 0.80,
                  hot_max_ratio: float = 0.25, hot_min_nodes: int = 256, add_self_loops: bool = True) -> dict:
    """graph_utils.py:174-241: the most-read nodes (covering a target share of
    all reads, within [min, max] nodes) moved to the front of `base_order`."""
    n = int(num_nodes)
    s = np.asarray(src, dtype=np.int64)
    if add_self_loops:
        s = np.concatenate([s, np.arange(n, dtype=np.int64)])
    access = np.bincount(s, minlength=n).astype(np.int64)
    order = _stable_desc(access)
    total = int(access.sum())
    cov = float(max(0.0, min(1.0, float(hot_access_coverage))))
    max_nodes = n if float(hot_max_ratio) <= 0.0 else max(1, min(n, int(np.ceil(float(hot_max_ratio) * n))))
    min_nodes = min(max(0, min(int(hot_min_nodes), n)), max_nodes)
    cutoff = min_nodes
    if total > 0 and cov > 0.0:
        prefix = np.cumsum(access[order])
        target = int(np.ceil(float(total) * cov))
        cutoff = max(cutoff, int(np.searchsorted(prefix, target, side="left")) + 1)
    elif total > 0:
        cutoff = max(cutoff, 1)
    cutoff = max(min_nodes, min(n, cutoff, max_nodes))
    hot_nodes = order[:cutoff].astype(np.int64)
    mask = np.zeros(n, bool)
    mask[hot_nodes] = True
    if base_order is None:
        perm = order.astype(np.int64)
    else:
        b = np.asarray(base_order, dtype=np.int64)
        perm = np.concatenate([b[mask[b]], b[~mask[b]]])
    inv = np.empty(n, np.int64)
    inv[perm] = np.arange(n, dtype=np.int64)
    hot_access = int(access[hot_nodes].sum()) if hot_nodes.size else 0
    return {
        "perm": perm, "inv_perm": inv, "hot_nodes": hot_nodes, "hot_node_cutoff": int(cutoff),
        "hot_node_fraction": float(cutoff / max(1, n)),
        "hot_node_access_coverage": float(hot_access / total) if total > 0 else 0.0,
        "hot_node_access_counts": access, "hot_total_accesses": total, "hot_access_target": cov,
        "hot_max_ratio": float(hot_max_ratio), "hot_min_nodes": int(min_nodes),
    }


def preprocess(src, dst, *, num_nodes: int, feat_dim: int = 128, page_bytes: int = 4096, row_block_size: int = 64,
               window_num_blocks: int = 4, window_cache_pages: int = 8, hot_cache_pages: int = 1024,
               signature_topk: int = 4, hot_access_coverage: float = 0.80, hot_max_ratio: float = 0.25,
               hot_min_nodes: int = 256) -> dict:
    """run/preprocess_gcn_graph.py:40-120: page schedule -> co-access order ->
    hot partition of that order -> renumbered graph -> its page schedule."""
    page_kw = dict(num_nodes=num_nodes, feat_dim=feat_dim, page_bytes=page_bytes, row_block_size=row_block_size,
                   hot_cache_pages=hot_cache_pages, signature_topk=signature_topk,
                   window_num_blocks=window_num_blocks, window_cache_pages=window_cache_pages)
    base = page_reuse_schedule(src, dst, **page_kw)
    perm, _ = coaccess_permutation(src, dst, num_nodes=num_nodes, row_schedule=base["row_schedule"],
                                   row_block_size=row_block_size, window_num_blocks=window_num_blocks,
                                   signature_topk=signature_topk)
    hot = hot_partition(src, num_nodes=num_nodes, base_order=perm, hot_access_coverage=hot_access_coverage,
                        hot_max_ratio=hot_max_ratio, hot_min_nodes=hot_min_nodes)
    inv = hot["inv_perm"]
    s_r = inv[np.asarray(src, dtype=np.int64)]
    d_r = inv[np.asarray(dst, dtype=np.int64)]
    final = page_reuse_schedule(s_r, d_r, **page_kw)
    return {"base": base, "coaccess_perm": perm, "hot": hot, "src": s_r, "dst": d_r, "final": final}
