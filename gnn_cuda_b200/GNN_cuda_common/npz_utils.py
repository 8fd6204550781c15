"""Graph loading in the reference's npz edge-list format (GNN_cuda_common/npz_utils.py).

An npz holds ``src_li`` and ``dst_li`` (edge endpoints) and optionally
``num_nodes`` and sparse features (``feat_indices`` [nnz, 2], ``feat_values``,
``feat_shape``). Without stored features the loaders draw N(0, 1) features from
PyTorch's global generator, like the reference (seed it with torch.manual_seed
for reproducible runs). ``save_graph_npz`` writes the same format.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch


def select_device(device_str: str) -> torch.device:
    if device_str.startswith("cuda") and not torch.cuda.is_available():
        return torch.device("cpu")
    return torch.device(device_str)


def _num_nodes(graph_obj) -> int:
    if "num_nodes" in graph_obj.files:
        return int(np.array(graph_obj["num_nodes"]).reshape(-1)[0])
    src = np.asarray(graph_obj["src_li"], dtype=np.int64)
    dst = np.asarray(graph_obj["dst_li"], dtype=np.int64)
    return max(int(src.max(initial=-1)), int(dst.max(initial=-1))) + 1


def _random_features(num_nodes: int, feat_dim: int) -> torch.Tensor:
    return torch.randn(num_nodes, feat_dim if feat_dim > 0 else 128, dtype=torch.float32)


def _stored_features(graph_obj, num_nodes: int, feat_dim: int) -> torch.Tensor:
    if not {"feat_indices", "feat_values", "feat_shape"}.issubset(set(graph_obj.files)):
        return _random_features(num_nodes, feat_dim)
    shape = np.asarray(graph_obj["feat_shape"]).astype(np.int64).reshape(-1)
    if shape.size != 2 or shape[0] <= 0 or shape[1] < 0:
        return _random_features(num_nodes, feat_dim)
    width = feat_dim if feat_dim > 0 else int(shape[1])
    width = width if width > 0 else 128
    feats = torch.zeros((num_nodes, width), dtype=torch.float32)
    idx = np.asarray(graph_obj["feat_indices"], dtype=np.int64)
    val = np.asarray(graph_obj["feat_values"], dtype=np.float32)
    if idx.ndim != 2 or idx.shape[1] != 2 or val.ndim != 1 or idx.shape[0] != val.shape[0]:
        return feats
    ok = (idx[:, 0] >= 0) & (idx[:, 0] < num_nodes) & (idx[:, 1] >= 0) & (idx[:, 1] < width)
    if ok.any():
        feats[torch.from_numpy(idx[ok, 0]), torch.from_numpy(idx[ok, 1])] = torch.from_numpy(val[ok])
    return feats


def _load_common(npz_path: str, feat_dim: int, use_npz_features: bool):
    path = Path(npz_path)
    if not path.exists():
        raise FileNotFoundError(f"graph file not found: {path}")
    g = np.load(str(path))
    src = np.asarray(g["src_li"], dtype=np.int64)
    dst = np.asarray(g["dst_li"], dtype=np.int64)
    n = _num_nodes(g)
    feats = _stored_features(g, n, feat_dim) if use_npz_features else _random_features(n, feat_dim)
    return src, dst, feats, n


def load_pyg_graph_features_from_npz(npz_path: str, feat_dim: int, use_npz_features: bool):
    src, dst, feats, n = _load_common(npz_path, feat_dim, use_npz_features)
    return torch.from_numpy(np.stack([src, dst], axis=0)).long(), feats, n


def load_dgl_graph_features_from_npz(npz_path: str, feat_dim: int, use_npz_features: bool):
    src, dst, feats, n = _load_common(npz_path, feat_dim, use_npz_features)
    return torch.from_numpy(src).long(), torch.from_numpy(dst).long(), feats, n


def save_graph_npz(path: str, src, dst, num_nodes: int) -> None:
    """Write an edge list in the reference's npz format."""
    np.savez(path, src_li=np.asarray(src, dtype=np.int64), dst_li=np.asarray(dst, dtype=np.int64),
             num_nodes=np.array([int(num_nodes)], dtype=np.int64))
