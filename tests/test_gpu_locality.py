"""Device locality preprocessing (gnn_locality_* through the graph_utils mirror)
against the reference's own outputs and the oracle, bit for bit.

Golden vectors: tests/golden/locality_cases.npz (the reference's
graph_utils.py:174-446 run on small graphs, chained as
run/preprocess_gcn_graph.py:40-120). Larger graphs: the oracle
(oracle/locality.py), itself pinned to those vectors by test_locality_oracle.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import locality as OL

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "locality_cases.npz"
PAGE_ARRAYS = ("page_histogram", "page_reuse_histogram", "hot_pages", "row_schedule", "block_hot_pages",
               "window_hot_pages")
PAGE_SCALARS = ("rows_per_page", "num_pages", "row_block_size", "window_num_blocks", "window_cache_pages",
                "rows_per_window", "signature_topk", "page_bytes", "hot_coverage", "avg_window_hot_coverage")
HOT_ARRAYS = ("perm", "inv_perm", "hot_nodes", "hot_node_access_counts")
HOT_SCALARS = ("hot_node_cutoff", "hot_total_accesses", "hot_min_nodes", "hot_node_fraction",
               "hot_node_access_coverage", "hot_access_target", "hot_max_ratio")


def _np(t):
    return t.cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def check_page(meta, exp_get, tag):
    for k in PAGE_ARRAYS:
        got, exp = _np(meta[k]), exp_get(k)
        assert got.shape == exp.shape and np.array_equal(got, exp), f"{tag}/{k}"
    for k in PAGE_SCALARS:
        assert float(meta[k]) == float(np.asarray(exp_get(k)).reshape(-1)[0]), f"{tag}/{k}"


def check_hot(hot, exp_get, tag):
    for k in HOT_ARRAYS:
        got, exp = _np(hot[k]), exp_get(k)
        assert got.shape == exp.shape and np.array_equal(got, exp), f"{tag}/{k}"
    for k in HOT_SCALARS:
        assert float(hot[k]) == float(np.asarray(exp_get(k)).reshape(-1)[0]), f"{tag}/{k}"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def _cases():
    return [str(c) for c in np.load(GOLDEN)["cases"]]


def _params(g, name):
    p = {k: int(g[f"{name}/param/{k}"][0]) for k in ("feat_dim", "page_bytes", "row_block_size", "window_num_blocks",
                                                     "window_cache_pages", "hot_cache_pages", "signature_topk",
                                                     "hot_min_nodes")}
    p.update({k: float(g[f"{name}/param/{k}"][0]) for k in ("hot_access_coverage", "hot_max_ratio")})
    return p


def _page_kw(p, n):
    return dict(num_nodes=n, feat_dim=p["feat_dim"], page_bytes=p["page_bytes"], row_block_size=p["row_block_size"],
                hot_cache_pages=p["hot_cache_pages"], signature_topk=p["signature_topk"],
                window_num_blocks=p["window_num_blocks"], window_cache_pages=p["window_cache_pages"])


@pytest.mark.parametrize("name", _cases())
def test_device_functions_match_reference(gold, name):
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    src, dst = torch.from_numpy(gold[f"{name}/src"]), torch.from_numpy(gold[f"{name}/dst"])
    n = int(gold[f"{name}/num_nodes"][0])
    p = _params(gold, name)
    # CPU inputs: computed on the GPU, returned on the CPU like the reference
    base = G.build_page_reuse_schedule_metadata(src, dst, **_page_kw(p, n))
    assert base["row_schedule"].device.type == "cpu"
    check_page(base, lambda k: gold[f"{name}/base/{k}"], f"{name}/base")
    perm, inv = G.build_coaccess_feature_permutation(src, dst, num_nodes=n, row_schedule=base["row_schedule"],
                                                     row_block_size=p["row_block_size"],
                                                     window_num_blocks=p["window_num_blocks"],
                                                     signature_topk=p["signature_topk"])
    assert np.array_equal(_np(perm), gold[f"{name}/coaccess/perm"])
    assert np.array_equal(_np(inv), gold[f"{name}/coaccess/inv_perm"])
    hot_kw = dict(num_nodes=n, hot_access_coverage=p["hot_access_coverage"], hot_max_ratio=p["hot_max_ratio"],
                  hot_min_nodes=p["hot_min_nodes"])
    hot = G.build_hot_partition_feature_permutation(src, base_order=perm, **hot_kw)
    check_hot(hot, lambda k: gold[f"{name}/hot/{k}"], f"{name}/hot")
    hot0 = G.build_hot_partition_feature_permutation(src, **hot_kw)
    check_hot(hot0, lambda k: gold[f"{name}/hot_nobase/{k}"], f"{name}/hot_nobase")


@pytest.mark.parametrize("name", _cases())
def test_device_pipeline_matches_reference(gold, name):
    from gnn_cuda_b200.GNN_cuda_common.locality import preprocess_gcn_graph
    dev = torch.device("cuda", 0)
    src = torch.from_numpy(gold[f"{name}/src"]).to(dev)
    dst = torch.from_numpy(gold[f"{name}/dst"]).to(dev)
    n = int(gold[f"{name}/num_nodes"][0])
    p = _params(gold, name)
    pay = preprocess_gcn_graph(src, dst, num_nodes=n, **p)
    assert pay["perm"].is_cuda  # device inputs keep device outputs
    check_hot(pay, lambda k: gold[f"{name}/hot/{k}"], f"{name}/payload-hot")
    check_page(pay, lambda k: gold[f"{name}/final/{k}"], f"{name}/payload-final")


def _rmat_edges(n, m, seed):
    rng = np.random.default_rng(seed)
    scale = int(np.ceil(np.log2(n)))
    s = np.zeros(m, np.int64)
    d = np.zeros(m, np.int64)
    for _ in range(scale):
        r = rng.random(m)
        s = 2 * s + (r >= 0.76)
        d = 2 * d + (((r >= 0.57) & (r < 0.76)) | (r >= 0.95))
    keep = (s < n) & (d < n)
    s, d = s[keep], d[keep]
    return np.concatenate([s, d]), np.concatenate([d, s])


@pytest.mark.parametrize("n,m,feat,rbs,wnb,wcp,k", [
    (50_000, 400_000, 128, 64, 4, 8, 4),
    (120_000, 900_000, 64, 32, 2, 12, 3),
])
def test_device_pipeline_matches_oracle_larger(n, m, feat, rbs, wnb, wcp, k):
    from gnn_cuda_b200.GNN_cuda_common.locality import preprocess_gcn_graph
    src, dst = _rmat_edges(n, m, seed=n + m)
    prm = dict(feat_dim=feat, row_block_size=rbs, window_num_blocks=wnb, window_cache_pages=wcp,
               hot_cache_pages=256, signature_topk=k, hot_access_coverage=0.8, hot_max_ratio=0.25, hot_min_nodes=256)
    ref = OL.preprocess(src, dst, num_nodes=n, **prm)
    dev = torch.device("cuda", 0)
    pay = preprocess_gcn_graph(torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev), num_nodes=n, **prm)
    check_hot(pay, lambda kk: np.asarray(ref["hot"][kk]), "hot")
    check_page(pay, lambda kk: np.asarray(ref["final"][kk]), "final")


def test_int32_row_ptr_schedule_matches_int64():
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    from gnn_cuda_b200.GNN_cuda_common.locality import page_schedule_from_csr
    dev = torch.device("cuda", 0)
    src, dst = _rmat_edges(20_000, 150_000, seed=5)
    s, d = torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev)
    out = []
    for dt in (torch.int32, torch.int64):
        rp, col, _ = G.device_csr(d, s, 20_000, True, dt, dev)
        out.append(page_schedule_from_csr(rp, col, num_nodes=20_000, rows_per_page=8))
    for key in PAGE_ARRAYS:
        assert torch.equal(out[0][key], out[1][key]), key
    ref = OL.page_reuse_schedule(src, dst, num_nodes=20_000, feat_dim=128)
    check_page(dict(out[0], page_bytes=4096), lambda kk: np.asarray(ref[kk]), "int32")


def test_bad_inputs_are_errors_and_device_stays_usable():
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    from gnn_cuda_b200.GNN_cuda_common.locality import apply_graph_permutation_device
    dev = torch.device("cuda", 0)
    src = torch.tensor([0, 1, 2, 7], device=dev)
    with pytest.raises(RuntimeError, match="outside"):
        G.build_hot_partition_feature_permutation(src, num_nodes=5)
    with pytest.raises(RuntimeError, match="permutation"):
        G.build_hot_partition_feature_permutation(src[:3], num_nodes=5,
                                                  base_order=torch.tensor([0, 1, 1, 3, 4], device=dev))
    with pytest.raises(ValueError):
        G.build_hot_partition_feature_permutation(src[:3], num_nodes=5, base_order=torch.arange(4, device=dev))
    inv = torch.arange(5, device=dev)
    with pytest.raises(RuntimeError, match="outside"):
        apply_graph_permutation_device(src, src, inv_perm=inv)
    # the context is still usable: a valid call right after succeeds
    hot = G.build_hot_partition_feature_permutation(src[:3], num_nodes=5, hot_min_nodes=1)
    assert hot["perm"].numel() == 5
    torch.cuda.synchronize()
