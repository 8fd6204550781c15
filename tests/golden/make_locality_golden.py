#!/usr/bin/env python3
"""Generate golden vectors for the UVM locality preprocessing by running the
reference's own host implementation.

Imports ``GNN_cuda_common/graph_utils.py`` from the reference checkout (read
only, in the development container; GPU test runs never run this) and records,
for small edge lists and several parameter sets, the outputs of
  build_page_reuse_schedule_metadata      (graph_utils.py:244-372)
  build_coaccess_feature_permutation      (graph_utils.py:375-446)
  build_hot_partition_feature_permutation (graph_utils.py:174-241)
  apply_graph_permutation                 (graph_utils.py:76-85)
chained exactly as run/preprocess_gcn_graph.py:40-120 chains them (page
schedule of the input graph -> co-access order -> hot prefix/cold suffix
partition of that order -> renumbered graph -> page schedule of the renumbered
graph), plus a hot partition without a base order. Everything goes into
``tests/golden/locality_cases.npz``; the tests check the oracle's restatement
(oracle/locality.py) and the device implementation against it bit for bit.

Usage:  python tests/golden/make_locality_golden.py [--reference DIR]  (default: $GNN_REFERENCE_ROOT, else ../reference)
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "locality_cases.npz"

# page-schedule keys the reference returns as tensors / ints / floats
TENSOR_KEYS = ("page_histogram", "page_reuse_histogram", "hot_pages", "row_schedule", "block_hot_pages",
               "window_hot_pages")
INT_KEYS = ("rows_per_page", "num_pages", "row_block_size", "window_num_blocks", "window_cache_pages",
            "rows_per_window", "signature_topk", "page_bytes")
FLOAT_KEYS = ("hot_coverage", "avg_window_hot_coverage")
HOT_TENSOR_KEYS = ("perm", "inv_perm", "hot_nodes", "hot_node_access_counts")
HOT_INT_KEYS = ("hot_node_cutoff", "hot_total_accesses", "hot_min_nodes")
HOT_FLOAT_KEYS = ("hot_node_fraction", "hot_node_access_coverage", "hot_access_target", "hot_max_ratio")


def _load_reference_graph_utils(reference: Path):
    path = reference / "GNN_cuda_common" / "graph_utils.py"
    spec = importlib.util.spec_from_file_location("reference_graph_utils", str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def _rmat(n: int, m: int, rng: np.random.Generator) -> tuple[np.ndarray, np.ndarray]:
    scale = max(1, int(np.ceil(np.log2(n))))
    s = np.zeros(m, np.int64)
    d = np.zeros(m, np.int64)
    for _ in range(scale):
        r = rng.random(m)
        s = 2 * s + (r >= 0.76)
        d = 2 * d + (((r >= 0.57) & (r < 0.76)) | (r >= 0.95))
    keep = (s < n) & (d < n)
    return s[keep], d[keep]


def _cases() -> dict[str, tuple[np.ndarray, np.ndarray, int, dict]]:
    rng = np.random.default_rng(20261202)
    cases = {}
    src = np.array([0, 2, 0, 2, 3, 4, 2, 1, 4, 0], dtype=np.int64)
    dst = np.array([1, 1, 1, 1, 3, 0, 1, 4, 2, 4], dtype=np.int64)
    small = dict(feat_dim=1024, row_block_size=2, window_num_blocks=2, window_cache_pages=2, hot_cache_pages=3,
                 signature_topk=2, hot_access_coverage=0.5, hot_max_ratio=0.5, hot_min_nodes=1)
    cases["handmade"] = (src, dst, 6, small)
    cases["single_node"] = (np.zeros(0, np.int64), np.zeros(0, np.int64), 1, {})
    cases["empty_edges"] = (np.zeros(0, np.int64), np.zeros(0, np.int64), 7, dict(hot_min_nodes=3))
    n = 300
    w = (np.arange(1, n + 1, dtype=np.float64)) ** (-1.0 / 1.1)
    p = w / w.sum()
    s = rng.choice(n, size=2500, p=p).astype(np.int64)
    d = rng.choice(n, size=2500, p=p).astype(np.int64)
    cases["powerlaw_default"] = (s, d, n, {})
    cases["powerlaw_f64_small_blocks"] = (s, d, n, dict(feat_dim=64, row_block_size=8, window_num_blocks=3,
                                                        window_cache_pages=5, hot_cache_pages=7, signature_topk=3,
                                                        hot_access_coverage=0.6, hot_max_ratio=0.1,
                                                        hot_min_nodes=4))
    cases["powerlaw_nocap"] = (s, d, n, dict(feat_dim=256, row_block_size=16, hot_access_coverage=1.0,
                                             hot_max_ratio=0.0, hot_min_nodes=0, signature_topk=1))
    cases["powerlaw_nocoverage"] = (s, d, n, dict(feat_dim=32, row_block_size=4, window_num_blocks=1,
                                                  window_cache_pages=1, hot_access_coverage=0.0, hot_min_nodes=5,
                                                  signature_topk=5))
    n2 = 1500
    s2 = np.concatenate([np.arange(1, n2), rng.integers(0, n2, 3000)]).astype(np.int64)
    d2 = np.concatenate([np.zeros(n2 - 1, np.int64), rng.integers(0, n2, 3000)]).astype(np.int64)
    cases["hub"] = (s2, d2, n2, dict(feat_dim=128, row_block_size=32, window_num_blocks=2, window_cache_pages=6,
                                     hot_cache_pages=20))
    u, v = _rmat(3000, 16000, rng)
    cases["rmat_sym"] = (np.concatenate([u, v]), np.concatenate([v, u]), 3000,
                         dict(feat_dim=128, row_block_size=64, window_num_blocks=4, window_cache_pages=8,
                              hot_cache_pages=64, signature_topk=4))
    return cases


DEFAULTS = dict(feat_dim=128, page_bytes=4096, row_block_size=64, window_num_blocks=4, window_cache_pages=8,
                hot_cache_pages=1024, signature_topk=4, hot_access_coverage=0.80, hot_max_ratio=0.25,
                hot_min_nodes=256)


def _record_page(arrays: dict, key: str, meta: dict) -> None:
    for k in TENSOR_KEYS:
        arrays[f"{key}/{k}"] = meta[k].numpy()
    for k in INT_KEYS:
        arrays[f"{key}/{k}"] = np.array([meta[k]], np.int64)
    for k in FLOAT_KEYS:
        arrays[f"{key}/{k}"] = np.array([meta[k]], np.float64)


def _record_hot(arrays: dict, key: str, hot: dict) -> None:
    for k in HOT_TENSOR_KEYS:
        arrays[f"{key}/{k}"] = hot[k].numpy()
    for k in HOT_INT_KEYS:
        arrays[f"{key}/{k}"] = np.array([hot[k]], np.int64)
    for k in HOT_FLOAT_KEYS:
        arrays[f"{key}/{k}"] = np.array([hot[k]], np.float64)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GNN_REFERENCE_ROOT",
                    str(Path(__file__).resolve().parents[3] / "reference")))
    args = ap.parse_args()
    gu = _load_reference_graph_utils(Path(args.reference))
    arrays: dict[str, np.ndarray] = {}
    names = []
    for name, (src, dst, n, over) in _cases().items():
        prm = dict(DEFAULTS, **over)
        names.append(name)
        s_t, d_t = torch.from_numpy(src), torch.from_numpy(dst)
        arrays[f"{name}/src"] = src
        arrays[f"{name}/dst"] = dst
        arrays[f"{name}/num_nodes"] = np.array([n], np.int64)
        for k, v in prm.items():
            arrays[f"{name}/param/{k}"] = np.array([v], np.float64 if isinstance(v, float) else np.int64)
        page_kw = dict(num_nodes=n, feat_dim=prm["feat_dim"], page_bytes=prm["page_bytes"],
                       row_block_size=prm["row_block_size"], hot_cache_pages=prm["hot_cache_pages"],
                       signature_topk=prm["signature_topk"], window_num_blocks=prm["window_num_blocks"],
                       window_cache_pages=prm["window_cache_pages"], add_self_loops=True)
        base = gu.build_page_reuse_schedule_metadata(s_t, d_t, **page_kw)
        _record_page(arrays, f"{name}/base", base)
        perm, inv_perm = gu.build_coaccess_feature_permutation(
            s_t, d_t, num_nodes=n, row_schedule=base["row_schedule"], row_block_size=prm["row_block_size"],
            window_num_blocks=prm["window_num_blocks"], signature_topk=prm["signature_topk"], add_self_loops=True)
        arrays[f"{name}/coaccess/perm"] = perm.numpy()
        arrays[f"{name}/coaccess/inv_perm"] = inv_perm.numpy()
        hot_kw = dict(num_nodes=n, hot_access_coverage=prm["hot_access_coverage"], hot_max_ratio=prm["hot_max_ratio"],
                      hot_min_nodes=prm["hot_min_nodes"], add_self_loops=True)
        hot = gu.build_hot_partition_feature_permutation(s_t, base_order=perm, **hot_kw)
        _record_hot(arrays, f"{name}/hot", hot)
        hot0 = gu.build_hot_partition_feature_permutation(s_t, base_order=None, **hot_kw)
        _record_hot(arrays, f"{name}/hot_nobase", hot0)
        s_r, d_r = gu.apply_graph_permutation(s_t, d_t, inv_perm=hot["inv_perm"])
        if src.size <= 10000:  # the renumbered edge list is inv_perm[src], inv_perm[dst]: kept for small cases only
            arrays[f"{name}/reordered/src"] = s_r.numpy()
            arrays[f"{name}/reordered/dst"] = d_r.numpy()
        final = gu.build_page_reuse_schedule_metadata(s_r, d_r, **page_kw)
        _record_page(arrays, f"{name}/final", final)
    arrays["cases"] = np.array(names)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays)} arrays, {len(names)} cases)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
