"""Memory-mapped npz reading (npz_utils.open_npz): same arrays as np.load, without reading members."""
import numpy as np
import torch

from gnn_cuda_b200.GNN_cuda_common import npz_utils as U


def test_open_npz_maps_stored_members_and_matches_np_load(tmp_path):
    rng = np.random.default_rng(3)
    src = rng.integers(0, 5000, 100_000).astype(np.int64)
    dst = rng.integers(0, 5000, 100_000).astype(np.int64)
    p = tmp_path / "g.npz"
    U.save_graph_npz(str(p), src, dst, 5000)
    g = U.open_npz(str(p))
    assert set(g.files) == {"src_li", "dst_li", "num_nodes"}
    assert isinstance(g["src_li"], np.memmap) and isinstance(g["dst_li"], np.memmap)
    ref = np.load(str(p))
    for k in ref.files:
        assert np.array_equal(np.asarray(g[k]), ref[k]) and g[k].dtype == ref[k].dtype


def test_open_npz_reads_compressed_and_fortran_members(tmp_path):
    p = tmp_path / "c.npz"
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    np.savez_compressed(str(p), a=a, empty=np.zeros((0, 2), np.int64))
    g = U.open_npz(str(p))
    assert np.array_equal(g["a"], a) and g["empty"].shape == (0, 2)
    q = tmp_path / "f.npz"
    np.savez(str(q), f=np.asfortranarray(a))
    assert np.array_equal(U.open_npz(str(q))["f"], a)


def test_loaders_on_mapped_npz_match_the_reference_format(tmp_path):
    src = np.array([0, 1, 2, 3], dtype=np.int64)
    dst = np.array([1, 2, 3, 0], dtype=np.int64)
    p = tmp_path / "tiny.npz"
    U.save_graph_npz(str(p), src, dst, 4)
    torch.manual_seed(0)
    ei, feats, n = U.load_pyg_graph_features_from_npz(str(p), 8, False)
    assert n == 4 and ei.dtype == torch.int64 and torch.equal(ei, torch.from_numpy(np.stack([src, dst])))
    s, d, f2, n2 = U.load_dgl_graph_features_from_npz(str(p), 8, False)
    s += 0  # tensors over copy-on-write pages are writable without touching the file
    assert torch.equal(s, torch.from_numpy(src)) and n2 == 4 and feats.shape == (4, 8)
    assert np.array_equal(np.load(str(p))["src_li"], src)
