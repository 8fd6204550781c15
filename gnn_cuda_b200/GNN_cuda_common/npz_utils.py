"""Graph loading in the reference's npz edge-list format (GNN_cuda_common/npz_utils.py).

An npz holds ``src_li`` and ``dst_li`` (edge endpoints) and optionally
``num_nodes`` and sparse features (``feat_indices`` [nnz, 2], ``feat_values``,
``feat_shape``). Without stored features the loaders draw N(0, 1) features from
PyTorch's global generator, like the reference (seed it with torch.manual_seed
for reproducible runs). ``save_graph_npz`` writes the same format, uncompressed,
and the loaders memory-map uncompressed members (``open_npz``) instead of
reading them, so billion-edge edge lists are paged in as they are used.
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


class MappedNpz:
    """Read-only view of an .npz whose stored (uncompressed) members are
    memory-mapped instead of read: a 1.6B-edge edge list costs page cache, not
    a private host copy, and a member is read only when it is touched.
    Compressed members are read normally. Same ``files`` / ``[]`` interface as
    ``np.load``'s NpzFile."""

    def __init__(self, path: str):
        import zipfile
        self.path = str(path)
        self._zip = zipfile.ZipFile(self.path)
        self._info = {i.filename[:-4] if i.filename.endswith(".npy") else i.filename: i
                      for i in self._zip.infolist()}
        self.files = list(self._info)

    def __contains__(self, key: str) -> bool:
        return key in self._info

    def __getitem__(self, key: str) -> np.ndarray:
        import zipfile
        info = self._info[key]
        if info.compress_type != zipfile.ZIP_STORED:
            with self._zip.open(info) as f:
                return np.lib.format.read_array(f, allow_pickle=False)
        with open(self.path, "rb") as raw:
            raw.seek(info.header_offset)
            local = raw.read(30)
            if local[:4] != b"PK\x03\x04":
                raise ValueError(f"{self.path}: bad local header for member {info.filename}")
            name_len = int.from_bytes(local[26:28], "little")
            extra_len = int.from_bytes(local[28:30], "little")
            data_start = info.header_offset + 30 + name_len + extra_len
            raw.seek(data_start)
            version = np.lib.format.read_magic(raw)
            if version == (1, 0):
                shape, fortran, dtype = np.lib.format.read_array_header_1_0(raw)
            else:
                shape, fortran, dtype = np.lib.format.read_array_header_2_0(raw)
            offset = raw.tell()
        if dtype.hasobject:
            raise ValueError(f"{self.path}: member {key} holds Python objects")
        count = int(np.prod(shape)) if shape else 1
        if count == 0:
            return np.zeros(shape, dtype=dtype)
        # copy-on-write: pages come from the file on first touch; a write stays private
        return np.memmap(self.path, dtype=dtype, mode="c", offset=offset, shape=shape,
                         order="F" if fortran else "C")

    def close(self) -> None:
        self._zip.close()


def open_npz(npz_path: str):
    """np.load-compatible reader that memory-maps uncompressed members."""
    return MappedNpz(npz_path)


def _load_common(npz_path: str, feat_dim: int, use_npz_features: bool):
    path = Path(npz_path)
    if not path.exists():
        raise FileNotFoundError(f"graph file not found: {path}")
    g = open_npz(str(path))
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
