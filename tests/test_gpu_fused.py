"""The fused aggregate-and-transform layer against the separate calls (run with -m gpu).

gnn_fused_aggregate_linear must return exactly what the reference's call
sequence returns on this library's TF32 tensor-core path:
  GCN   spmm_gcn_forward_ -> linear_forward_(relu?)           (gcn_inference.py:534-600)
  GIN   spmm_sum_forward_ -> tensor_add_inplace_(1 + eps) -> linear_forward_(relu)
        -> linear_forward_(relu?)                             (gin_inference.py:317-359)
  mean  spmm_mean_forward_ -> linear_forward_(relu?)
on graphs with power-law hubs, with the long-row threshold forced low so that
single- and multi-segment long rows (summed before the transform and written
back into their output rows) are exercised. The comparison is bit for bit;
each case is also held to the TF32 tolerance (2e-3 of sum |a w|) against a
float64 transform of the oracle's aggregate.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200 import _native as N
from gnn_cuda_b200 import synth
from gnn_cuda_b200.GNN_cuda_common import agg_ops, fused_ops, gcn_ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _tf32_and_threshold():
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    old_thr = N.config_get("spmm.long_row_threshold")
    torch.backends.cuda.matmul.allow_tf32 = True
    yield
    torch.backends.cuda.matmul.allow_tf32 = old_tf32
    N.config_set("spmm.long_row_threshold", old_thr)


def _hub_graph(n: int, seed: int, hubs=(0, 1, 2), loops=True, index=torch.int32):
    g = torch.Generator().manual_seed(seed)
    u, v = synth.rmat_undirected(n, n * 6, seed=seed)
    # a few hub rows: degree ~n/2 (multi-segment at a low threshold) and ~n/8
    extra_u, extra_v = [], []
    for k, h in enumerate(hubs):
        m = n // (2 if k == 0 else 8)
        extra_u.append(torch.full((m,), h, dtype=torch.int64))
        extra_v.append(torch.randint(0, n, (m,), generator=g))
    u = torch.cat([u] + extra_u)
    v = torch.cat([v] + extra_v)
    keep = u != v
    key = torch.unique(torch.minimum(u[keep], v[keep]) * n + torch.maximum(u[keep], v[keep]))
    s, d = synth.symmetrize(key // n, key % n)
    rp, ci, dis = synth.csr_on_device(s, d, n, add_self_loops=loops, index_dtype=index)
    return rp.to(DEV), ci.to(DEV), dis.to(DEV)


def _bits(t):
    return t.detach().cpu().numpy().view(np.uint32)


def _tf32_err(got, a, w, b, relu):
    a = a.astype(np.float64)
    exp = a @ w.astype(np.float64) + (0 if b is None else b.astype(np.float64))
    if relu:
        exp = np.maximum(exp, 0)
    scale = np.abs(a) @ np.abs(w.astype(np.float64)) + (0 if b is None else np.abs(b)) + 1e-30
    return float(np.max(np.abs(got.astype(np.float64) - exp) / scale))


@pytest.mark.parametrize("n,k,width,thr,relu,bias", [
    (20000, 128, 128, 64, True, True),
    (20000, 128, 128, 0, False, False),
    (5000, 64, 128, 40, True, True),
    (3001, 32, 64, 40, False, True),
    (777, 96, 128, 32, True, True),
])
def test_gcn_layer_bit_exact_vs_separate_calls(n, k, width, thr, relu, bias):
    N.config_set("spmm.long_row_threshold", thr)
    rp, ci, dis = _hub_graph(n, seed=n + k)
    x = synth.features(n, k, seed=3, device=DEV)
    w = synth.glorot(k, width, seed=4, device=DEV)
    b = torch.randn(width, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV) if bias else None
    agg = torch.empty(n, k, device=DEV)
    gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, agg)
    ref = torch.empty(n, width, device=DEV)
    agg_ops.linear_forward_(agg, w, b, ref, relu)
    assert fused_ops.fused_supported(k, width)
    out = torch.full((n, width), float("nan"), device=DEV)
    fused_ops.gcn_layer_forward_(rp, ci, dis, x, w, b, out, relu)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), _bits(ref))
    # and against float64 of the oracle's aggregate
    exp_agg = O.spmm(rp.cpu().numpy(), ci.cpu().numpy(), x.cpu().numpy(), mode=O.W_GCN, dis=dis.cpu().numpy(),
                     split_warps=16, long_thr=thr if thr else 256)
    assert np.array_equal(_bits(agg), exp_agg.view(np.uint32))
    assert _tf32_err(out.cpu().numpy(), exp_agg, w.cpu().numpy(), None if b is None else b.cpu().numpy(),
                     relu) <= 2e-3


@pytest.mark.parametrize("eps,relu_out,index", [(0.0, True, torch.int32), (0.25, False, torch.int32),
                                                (0.0, False, torch.int64)])
def test_gin_layer_bit_exact_vs_separate_calls(eps, relu_out, index):
    N.config_set("spmm.long_row_threshold", 48)
    n, f = 12000, 128
    rp, ci, _ = _hub_graph(n, seed=11, loops=False, index=index)
    x = synth.features(n, f, seed=12, device=DEV)
    w1 = synth.glorot(f, f, seed=13, device=DEV)
    w2 = synth.glorot(f, f, seed=14, device=DEV)
    b1 = torch.randn(f, generator=torch.Generator(device=DEV).manual_seed(15), device=DEV)
    b2 = torch.randn(f, generator=torch.Generator(device=DEV).manual_seed(16), device=DEV)
    agg = torch.empty(n, f, device=DEV)
    hid = torch.empty(n, f, device=DEV)
    ref = torch.empty(n, f, device=DEV)
    agg_ops.spmm_sum_forward_(rp, ci, x, agg)
    agg_ops.tensor_add_inplace_(agg, x, 1.0 + eps)
    agg_ops.linear_forward_(agg, w1, b1, hid, True)
    agg_ops.linear_forward_(hid, w2, b2, ref, relu_out)
    out = torch.full((n, f), float("nan"), device=DEV)
    fused_ops.gin_layer_forward_(rp, ci, x, eps, w1, b1, w2, b2, out, relu_out)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), _bits(ref))


@pytest.mark.parametrize("reciprocal", [False, True])
def test_mean_layer_bit_exact_vs_separate_calls(reciprocal):
    N.config_set("spmm.long_row_threshold", 40)
    n, f = 9000, 128
    rp, ci, _ = _hub_graph(n, seed=21, loops=False)
    x = synth.features(n, f, seed=22, device=DEV)
    w = synth.glorot(f, f, seed=23, device=DEV)
    b = torch.randn(f, generator=torch.Generator(device=DEV).manual_seed(24), device=DEV)
    agg = torch.empty(n, f, device=DEV)
    ref = torch.empty(n, f, device=DEV)
    agg_ops.spmm_mean_forward_(rp, ci, x, agg, hmm_optimized=reciprocal)
    agg_ops.linear_forward_(agg, w, b, ref, True)
    out = torch.full((n, f), float("nan"), device=DEV)
    fused_ops.mean_linear_forward_(rp, ci, x, w, b, out, True, reciprocal)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), _bits(ref))


def test_edge_cases_small_and_empty_graphs():
    """1 node, rows past the last full tile, a graph with no entries, isolated rows."""
    for n, pairs in ((1, 0), (5, 3), (130, 200), (300, 0)):
        w = synth.glorot(128, 128, seed=31, device=DEV)
        b = torch.randn(128, generator=torch.Generator(device=DEV).manual_seed(32), device=DEV)
        if pairs:
            u, v = synth.rmat_undirected(n, pairs, seed=33)
            s, d = synth.symmetrize(u, v)
        else:
            s = d = torch.zeros(0, dtype=torch.int64)
        rp, ci, dis = synth.csr_on_device(s, d, n, add_self_loops=False)
        rp, ci, dis = rp.to(DEV), ci.to(DEV), dis.to(DEV)
        x = synth.features(n, 128, seed=34, device=DEV)
        agg = torch.empty(n, 128, device=DEV)
        ref = torch.empty(n, 128, device=DEV)
        gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, agg)
        agg_ops.linear_forward_(agg, w, b, ref, True)
        out = torch.full((n, 128), float("nan"), device=DEV)
        fused_ops.gcn_layer_forward_(rp, ci, dis, x, w, b, out, True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(out), _bits(ref)), n


def test_refusals():
    L = N.lib()
    assert L.gnn_fused_layer_supported(256, 128, 0) == 0    # feat_dim above 128
    assert L.gnn_fused_layer_supported(128, 64, 0) == 0     # output narrower than feat_dim
    assert L.gnn_fused_layer_supported(128, 128, 48) == 0   # width not 32 / 64 / 128
    assert L.gnn_fused_layer_supported(128, 128, 128) == 1
    n = 100
    x = torch.zeros(n, 128, device=DEV)
    rp = torch.zeros(n + 1, dtype=torch.int32, device=DEV)
    ci = torch.zeros(0, dtype=torch.int32, device=DEV)
    w = torch.zeros(128, 128, device=DEV)
    with pytest.raises(RuntimeError, match="alias"):
        fused_ops.gcn_layer_forward_(rp, ci, torch.ones(n, device=DEV), x, w, None, x, False)
    out = torch.zeros(n, 128, device=DEV)
    rc = L.gnn_fused_aggregate_linear(ctypes.c_void_p(rp.data_ptr()), 0, None, None, 7, 0,
                                      ctypes.c_void_p(x.data_ptr()), n, n, 0, 128, 1.0, 0,
                                      ctypes.c_void_p(w.data_ptr()), None, 128, 0, None, None, 0, 0,
                                      ctypes.c_void_p(out.data_ptr()), None, 0, None)
    assert rc == 1 and "aggregation must be" in N.last_error()


@pytest.mark.parametrize("chunks", [1, 3, 16])
def test_gin_row_chunks_bit_exact_vs_separate_calls(chunks):
    """The GIN layer run as the separate calls over row ranges (gin_layer_row_chunks_)
    equals the whole-graph calls bit for bit, hub rows included."""
    N.config_set("spmm.long_row_threshold", 0)
    n, f = 12000, 128
    rp, ci, _ = _hub_graph(n, seed=41, loops=False, index=torch.int64)
    x = synth.features(n, f, seed=42, device=DEV)
    w1 = synth.glorot(f, f, seed=43, device=DEV)
    w2 = synth.glorot(f, f, seed=44, device=DEV)
    b1 = torch.randn(f, generator=torch.Generator(device=DEV).manual_seed(45), device=DEV)
    b2 = torch.randn(f, generator=torch.Generator(device=DEV).manual_seed(46), device=DEV)
    agg = torch.empty(n, f, device=DEV)
    hid = torch.empty(n, f, device=DEV)
    ref = torch.empty(n, f, device=DEV)
    agg_ops.spmm_sum_forward_(rp, ci, x, agg)
    agg_ops.tensor_add_inplace_(agg, x, 1.0)
    agg_ops.linear_forward_(agg, w1, b1, hid, True)
    agg_ops.linear_forward_(hid, w2, b2, ref, True)
    out = torch.full((n, f), float("nan"), device=DEV)
    fused_ops.gin_layer_row_chunks_(rp, ci, x, 0.0, w1, b1, w2, b2, out, True, chunks=chunks)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), _bits(ref))
    assert N.config_get("spmm.long_row_threshold") == 0  # restored
