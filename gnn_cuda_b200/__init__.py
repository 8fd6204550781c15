"""gnn_cuda_b200 — B200-native (sm_100a) engine for the GNN aggregation hot path.

``gnn_cuda_b200.GNN_cuda_common`` mirrors the operator surface of
jonghyun1215/GNN_cuda's ``GNN_cuda_common`` package (agg_ops, gcn_ops,
pyg_gcn_ops, allocator, loader, graph_utils and the three model drivers); the
kernels live in ``libgnnb200.so`` behind the C ABI in ``include/gnn_b200.h``.
"""
__version__ = "0.1.0"
