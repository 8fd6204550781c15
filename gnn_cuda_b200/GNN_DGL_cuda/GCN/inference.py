#!/usr/bin/env python3
"""GCN inference, dgl label (reference: GNN_DGL_cuda/GCN/inference.py)."""
from gnn_cuda_b200.GNN_cuda_common.gcn_inference import run_gcn_inference
from gnn_cuda_b200.GNN_cuda_common.npz_utils import load_dgl_graph_features_from_npz, select_device


def main() -> int:
    return run_gcn_inference(framework_label="dgl", select_device=select_device,
                             load_graph_features=load_dgl_graph_features_from_npz, load_kind="dgl")


if __name__ == "__main__":
    raise SystemExit(main())
