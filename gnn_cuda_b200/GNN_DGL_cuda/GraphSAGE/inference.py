#!/usr/bin/env python3
"""GraphSAGE inference, dgl label (reference: GNN_DGL_cuda/GraphSAGE/inference.py)."""
from gnn_cuda_b200.GNN_cuda_common.graphsage_inference import run_graphsage_inference
from gnn_cuda_b200.GNN_cuda_common.npz_utils import load_dgl_graph_features_from_npz, select_device


def main() -> int:
    return run_graphsage_inference(framework_label="dgl", select_device=select_device,
                                   load_graph_features=load_dgl_graph_features_from_npz, load_kind="dgl")


if __name__ == "__main__":
    raise SystemExit(main())
