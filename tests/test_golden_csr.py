"""CSR construction pinned bit for bit against the reference's own builders.

The golden arrays in tests/golden/csr_cases.npz were produced by running the
reference's graph_utils.build_* functions (tests/golden/make_golden.py). Both
the oracle's restatement and this package's sort-based builders must equal
them exactly: row_ptr, col_ind, deg_inv_sqrt and edge_weight.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200.GNN_cuda_common import graph_utils as G

CASES = ["handmade", "single_node", "single_node_selfloop", "empty_edges", "powerlaw_dups", "hub"]


def _case(golden, name):
    return golden[f"{name}/src"], golden[f"{name}/dst"], int(golden[f"{name}/num_nodes"][0])


def _eq(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    assert a.dtype == b.dtype, (a.dtype, b.dtype)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.array_equal(a.view(np.uint8) if a.dtype.kind == "f" else a, b.view(np.uint8) if b.dtype.kind == "f" else b)


@pytest.mark.parametrize("name", CASES)
def test_oracle_gcn_csr_matches_reference(golden, name):
    s, d, n = _case(golden, name)
    for loops, key in ((True, "gcn"), (False, "gcn_noloops")):
        rp, ci, dis = O.gcn_normalized_csr(s, d, n, add_self_loops=loops)
        _eq(rp, golden[f"{name}/{key}/row_ptr"])
        _eq(ci, golden[f"{name}/{key}/col_ind"])
        _eq(dis, golden[f"{name}/{key}/deg_inv_sqrt"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_pyg_and_plain_match_reference(golden, name):
    s, d, n = _case(golden, name)
    rp, ci, ew = O.pyg_weighted_csr(s, d, n)
    _eq(rp, golden[f"{name}/pyg/row_ptr"])
    _eq(ci, golden[f"{name}/pyg/col_ind"])
    _eq(ew, golden[f"{name}/pyg/edge_weight"])
    for loops in (0, 1):
        for tr in (0, 1):
            rp, ci = O.plain_csr(s, d, n, add_self_loops=bool(loops), transpose_for_incoming=bool(tr))
            _eq(rp, golden[f"{name}/plain_l{loops}_t{tr}/row_ptr"])
            _eq(ci, golden[f"{name}/plain_l{loops}_t{tr}/col_ind"])


@pytest.mark.parametrize("name", CASES)
def test_package_builders_match_reference(golden, name):
    s, d, n = _case(golden, name)
    st, dt = torch.from_numpy(s), torch.from_numpy(d)
    g = G.build_gcn_normalized_csr(st, dt, num_nodes=n, add_self_loops=True)
    _eq(g.row_ptr.numpy(), golden[f"{name}/gcn/row_ptr"])
    _eq(g.col_ind.numpy(), golden[f"{name}/gcn/col_ind"])
    _eq(g.deg_inv_sqrt.numpy(), golden[f"{name}/gcn/deg_inv_sqrt"])
    assert g.num_edges == golden[f"{name}/gcn/col_ind"].shape[0] and g.num_nodes == n
    w = G.build_pyg_gcn_weighted_csr(st, dt, num_nodes=n)
    _eq(w.row_ptr.numpy(), golden[f"{name}/pyg/row_ptr"])
    _eq(w.col_ind.numpy(), golden[f"{name}/pyg/col_ind"])
    _eq(w.edge_weight.numpy(), golden[f"{name}/pyg/edge_weight"])
    for loops in (0, 1):
        for tr in (0, 1):
            p = G.build_plain_csr(st, dt, num_nodes=n, add_self_loops=bool(loops), transpose_for_incoming=bool(tr))
            _eq(p.row_ptr.numpy(), golden[f"{name}/plain_l{loops}_t{tr}/row_ptr"])
            _eq(p.col_ind.numpy(), golden[f"{name}/plain_l{loops}_t{tr}/col_ind"])


def test_int64_row_ptr_option(golden):
    s, d, n = _case(golden, "powerlaw_dups")
    g = G.build_gcn_normalized_csr(torch.from_numpy(s), torch.from_numpy(d), num_nodes=n, index_dtype=torch.int64)
    assert g.row_ptr.dtype == torch.int64
    assert np.array_equal(g.row_ptr.numpy(), golden["powerlaw_dups/gcn/row_ptr"].astype(np.int64))


def test_out_of_range_ids_raise():
    with pytest.raises(ValueError):
        G.build_plain_csr(torch.tensor([0, 5]), torch.tensor([1, 2]), num_nodes=3)
    with pytest.raises(ValueError):
        G.build_plain_csr(torch.tensor([0, -1]), torch.tensor([1, 2]), num_nodes=3)


def test_device_csr_builder_matches_host_builder():
    from gnn_cuda_b200 import synth
    u, v = synth.rmat_undirected(5000, 20000, seed=3)
    s, d = synth.symmetrize(u, v)
    rp, ci, dis = synth.csr_on_device(s, d, 5000, add_self_loops=True)
    g = G.build_gcn_normalized_csr(s, d, num_nodes=5000)
    assert torch.equal(rp, g.row_ptr)
    assert torch.equal(ci, g.col_ind)
    assert torch.equal(dis.view(torch.int32), g.deg_inv_sqrt.view(torch.int32))
