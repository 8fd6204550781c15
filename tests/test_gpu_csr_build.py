"""Device CSR builder (gnn_csr_build) against the reference's golden CSR arrays and
the host builders, bit for bit (run with -m gpu).

The golden arrays in tests/golden/csr_cases.npz come from running the
reference's own graph_utils builders (tests/golden/make_golden.py); CUDA inputs
to graph_utils.build_* take the device path and must reproduce them exactly.
"""
import numpy as np
import pytest
import torch

from gnn_cuda_b200 import synth
from gnn_cuda_b200.GNN_cuda_common import graph_utils as G

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
CASES = ["handmade", "single_node", "single_node_selfloop", "empty_edges", "powerlaw_dups", "hub"]


def _eq(got: torch.Tensor, want) -> None:
    g = got.cpu().numpy()
    w = np.asarray(want)
    assert g.dtype == w.dtype and g.shape == w.shape, (g.dtype, w.dtype, g.shape, w.shape)
    assert np.array_equal(g.view(np.uint8), w.view(np.uint8))


@pytest.mark.parametrize("name", CASES)
def test_device_builders_match_reference_golden(golden, name):
    s = torch.from_numpy(golden[f"{name}/src"]).to(DEV)
    d = torch.from_numpy(golden[f"{name}/dst"]).to(DEV)
    n = int(golden[f"{name}/num_nodes"][0])
    for loops, key in ((True, "gcn"), (False, "gcn_noloops")):
        g = G.build_gcn_normalized_csr(s, d, num_nodes=n, add_self_loops=loops)
        assert g.row_ptr.is_cuda and g.col_ind.is_cuda and g.deg_inv_sqrt.is_cuda
        _eq(g.row_ptr, golden[f"{name}/{key}/row_ptr"])
        _eq(g.col_ind, golden[f"{name}/{key}/col_ind"])
        _eq(g.deg_inv_sqrt, golden[f"{name}/{key}/deg_inv_sqrt"])
        assert g.num_edges == golden[f"{name}/{key}/col_ind"].shape[0]
    w = G.build_pyg_gcn_weighted_csr(s, d, num_nodes=n)
    _eq(w.row_ptr, golden[f"{name}/pyg/row_ptr"])
    _eq(w.col_ind, golden[f"{name}/pyg/col_ind"])
    _eq(w.edge_weight, golden[f"{name}/pyg/edge_weight"])
    for loops in (0, 1):
        for tr in (0, 1):
            p = G.build_plain_csr(s, d, num_nodes=n, add_self_loops=bool(loops), transpose_for_incoming=bool(tr))
            _eq(p.row_ptr, golden[f"{name}/plain_l{loops}_t{tr}/row_ptr"])
            _eq(p.col_ind, golden[f"{name}/plain_l{loops}_t{tr}/col_ind"])


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_device_builder_matches_host_on_rmat(index_dtype):
    n = 300_000
    u, v = synth.rmat_undirected(n, n * 10, seed=41)
    s, d = synth.symmetrize(u, v)
    # duplicates and existing self-loops on purpose
    s = torch.cat([s, s[:1000], torch.arange(0, 50)])
    d = torch.cat([d, d[:1000], torch.arange(0, 50)])
    host = G.build_pyg_gcn_weighted_csr(s, d, num_nodes=n, index_dtype=index_dtype)
    dev = G.build_pyg_gcn_weighted_csr(s.to(DEV), d.to(DEV), num_nodes=n, index_dtype=index_dtype)
    _eq(dev.row_ptr, host.row_ptr.numpy())
    _eq(dev.col_ind, host.col_ind.numpy())
    _eq(dev.edge_weight, host.edge_weight.numpy())
    gh = G.build_gcn_normalized_csr(s, d, num_nodes=n)
    gd = G.build_gcn_normalized_csr(s.to(DEV), d.to(DEV), num_nodes=n)
    _eq(gd.deg_inv_sqrt, gh.deg_inv_sqrt.numpy())
    # int32 ids on the device are accepted too
    g32 = G.build_plain_csr(s.to(DEV, torch.int32), d.to(DEV, torch.int32), num_nodes=n)
    p = G.build_plain_csr(s, d, num_nodes=n)
    _eq(g32.row_ptr, p.row_ptr.numpy())
    _eq(g32.col_ind, p.col_ind.numpy())


@pytest.mark.parametrize("bad,msg", [((-1, 0), "negative column index found"),
                                     ((0, -2), "negative row index found"),
                                     ((5, 0), "column index exceeds matrix dimensions"),
                                     ((0, 5), "row index exceeds matrix dimensions")])
def test_device_builder_rejects_out_of_range_ids_like_host(bad, msg):
    n = 5
    s = torch.tensor([0, 1, bad[0]], dtype=torch.int64)
    d = torch.tensor([1, 2, bad[1]], dtype=torch.int64)
    with pytest.raises(ValueError, match=msg):
        G.build_gcn_normalized_csr(s, d, num_nodes=n, add_self_loops=False)
    with pytest.raises(ValueError, match=msg):
        G.build_gcn_normalized_csr(s.to(DEV), d.to(DEV), num_nodes=n, add_self_loops=False)
