#!/usr/bin/env python3
"""GCN locality preprocessing for ``--spmm_mode optimized`` (reference:
run/preprocess_gcn_graph.py), computed on the GPU.

Same flags, defaults, output file (``<data_root>/gnn_cuda_preprocessed/gcn/
<dataset>.pt``), payload keys and report lines as the reference script. The
chain is the reference's — page schedule of the graph, co-access node order,
hot-prefix partition of that order, renumbered graph, page schedule of the
renumbered graph — run by ``locality.preprocess_gcn_graph`` on one CUDA
device, bit for bit the reference's arrays.

  python -m gnn_cuda_b200.run.preprocess_gcn_graph --dataset NAME [--data_root DIR] [...]
"""
from __future__ import annotations

import argparse
import os
import time
from pathlib import Path

import numpy as np
import torch

from gnn_cuda_b200.GNN_cuda_common.graph_utils import default_gcn_preprocess_meta_path, resolve_dataset_path
from gnn_cuda_b200.GNN_cuda_common.locality import preprocess_gcn_graph

DEFAULT_DATA_ROOT = os.environ.get("GNN_DATASET_ROOT", "/root/workspace/mnt/dataset_npz")


def _load_edges(npz_path: str) -> tuple[torch.Tensor, torch.Tensor, int]:
    g = np.load(npz_path)
    src = torch.from_numpy(np.asarray(g["src_li"], dtype=np.int64))
    dst = torch.from_numpy(np.asarray(g["dst_li"], dtype=np.int64))
    if "num_nodes" in g.files:
        n = int(np.asarray(g["num_nodes"]).reshape(-1)[0])
    else:
        n = max(int(src.max()), int(dst.max())) + 1
    return src, dst, n


def preprocess_one(dataset: str, *, data_root: str, device: torch.device, **params) -> Path:
    graph_path = resolve_dataset_path(dataset, data_root=data_root)
    src, dst, num_nodes = _load_edges(graph_path)
    t0 = time.perf_counter()
    payload = preprocess_gcn_graph(src.to(device), dst.to(device), num_nodes=num_nodes, **params)
    torch.cuda.synchronize(device)
    elapsed = time.perf_counter() - t0
    payload = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in payload.items()}
    payload = {"dataset": dataset, "graph_path": str(graph_path), **payload}
    out_path = Path(default_gcn_preprocess_meta_path(dataset, data_root=data_root))
    out_path.parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, out_path)
    print(f"Saved GCN preprocess metadata: {out_path}")
    print(
        f"dataset={dataset} nodes={num_nodes} num_pages={payload['num_pages']} "
        f"hot_pages={int(payload['hot_pages'].numel())} hot_coverage={float(payload['hot_coverage']):.6f} "
        f"hot_nodes={int(payload['hot_node_cutoff'])} hot_node_fraction={float(payload['hot_node_fraction']):.6f} "
        f"hot_node_access_coverage={float(payload['hot_node_access_coverage']):.6f} "
        f"rows_per_page={int(payload['rows_per_page'])} row_block_size={int(payload['row_block_size'])} "
        f"window_num_blocks={int(payload['window_num_blocks'])} "
        f"window_cache_pages={int(payload['window_cache_pages'])} "
        f"avg_window_hot_coverage={float(payload['avg_window_hot_coverage']):.6f}"
    )
    reuse = payload["page_reuse_histogram"]
    bins = torch.nonzero(reuse, as_tuple=False).flatten()
    if int(bins.numel()) > 0:
        head = bins[:8].tolist()
        print("page_reuse_histogram=" + ", ".join(f"{int(b)}->{int(reuse[int(b)])}" for b in head))
    print(f"preprocess_gpu_seconds={elapsed:.3f} device={device}")
    return out_path


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--dataset", type=str, required=True, help="dataset name or all")
    p.add_argument("--data_root", type=str, default=DEFAULT_DATA_ROOT, help="directory containing <dataset>.npz")
    p.add_argument("--feat_dim", type=int, default=128, help="feature dimension used for page packing")
    p.add_argument("--page_bytes", type=int, default=4096, help="logical host page size for page reuse packing")
    p.add_argument("--row_block_size", type=int, default=64, help="destination rows per packed block")
    p.add_argument("--window_num_blocks", type=int, default=4, help="number of row-blocks per staged hot-page window")
    p.add_argument("--window_cache_pages", type=int, default=8, help="pages staged per row-block window")
    p.add_argument("--hot_cache_pages", type=int, default=1024, help="number of hot feature pages to stage on the GPU")
    p.add_argument("--signature_topk", type=int, default=4, help="number of dominant pages per row signature")
    p.add_argument("--hot_access_coverage", type=float, default=0.80,
                   help="target source-access coverage for the staged hot-node prefix")
    p.add_argument("--hot_max_ratio", type=float, default=0.25,
                   help="maximum node fraction that can be promoted into the hot prefix")
    p.add_argument("--hot_min_nodes", type=int, default=256, help="minimum node count in the hot prefix")
    p.add_argument("--device", type=str, default="cuda:0", help="CUDA device that runs the preprocessing")
    args = p.parse_args(argv)
    datasets = (sorted(q.stem for q in Path(args.data_root).glob("*.npz")) if args.dataset == "all"
                else [str(args.dataset)])
    if not datasets:
        raise FileNotFoundError(f"no .npz datasets found in: {args.data_root}")
    device = torch.device(args.device)
    params = dict(feat_dim=args.feat_dim, page_bytes=args.page_bytes, row_block_size=args.row_block_size,
                  window_num_blocks=args.window_num_blocks, window_cache_pages=args.window_cache_pages,
                  hot_cache_pages=args.hot_cache_pages, signature_topk=args.signature_topk,
                  hot_access_coverage=args.hot_access_coverage, hot_max_ratio=args.hot_max_ratio,
                  hot_min_nodes=args.hot_min_nodes)
    for ds in datasets:
        preprocess_one(ds, data_root=args.data_root, device=device, **params)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
