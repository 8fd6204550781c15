"""The C oracle against independent restatements (CPU only).

* sum / mean are checked against a pure-Python float32 loop in CSR order on a
  small graph (exact: float32 additions in the same order give the same bits);
* every mode is checked against the float64 aggregation within the
  fp32 tolerance |ours - f64| <= 1e-5 * (sum|terms| + |f64|);
* the long-row split schedule equals plain CSR order on rows below the
  threshold, and stays within the same tolerance above it.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200 import synth


@pytest.fixture(scope="module")
def graph():
    u, v = synth.chung_lu_undirected(600, 2500, max_degree=120.0, seed=11)
    s, d = synth.symmetrize(u, v)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), 600)
    _, _, ew = O.pyg_weighted_csr(s.numpy(), d.numpy(), 600)
    x = synth.features(600, 24, seed=5).numpy()
    return rp, ci, dis, ew, x


def _py_sum(rp, ci, x, mean):
    out = np.zeros_like(x)
    for r in range(len(rp) - 1):
        acc = [np.float32(0.0)] * x.shape[1]
        for e in range(rp[r], rp[r + 1]):
            row = x[ci[e]]
            acc = [np.float32(a + row[j]) for j, a in enumerate(acc)]
        deg = rp[r + 1] - rp[r]
        if mean == O.M_DIV and deg:
            acc = [np.float32(a / np.float32(deg)) for a in acc]
        if mean == O.M_RCP and deg:
            inv = np.float32(np.float32(1.0) / np.float32(deg))
            acc = [np.float32(a * inv) for a in acc]
        out[r] = acc
    return out


@pytest.mark.parametrize("mean", [O.M_NONE, O.M_DIV, O.M_RCP])
def test_sum_mean_bit_exact_vs_python_loop(graph, mean):
    rp, ci, _, _, x = graph
    rp_s = rp[:121]  # first 120 rows keep the Python loop short
    ours = O.spmm(rp, ci, x, mode=O.W_UNIT, mean=mean, rows=(0, 120))
    ref = _py_sum(rp_s, ci, x, mean)[:120]
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("mode", [O.W_UNIT, O.W_GCN, O.W_EDGE])
def test_oracle_within_f64_tolerance(graph, mode):
    rp, ci, dis, ew, x = graph
    ours = O.spmm(rp, ci, x, mode=mode, dis=dis, ew=ew)
    ref, ab = O.spmm_f64(rp, ci, x, mode=mode, dis=dis, ew=ew)
    assert O.check_close_to_f64(ours, ref, ab) <= 1.0


def test_gcn_equals_pyg_weighted(graph):
    """dis[r]*dis[c] computed on the fly equals the precomputed edge weight: same bits."""
    rp, ci, dis, ew, x = graph
    a = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis)
    b = O.spmm(rp, ci, x, mode=O.W_EDGE, ew=ew)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_split_schedule(graph):
    rp, ci, dis, _, x = graph
    thr = 40
    seq = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis)
    split = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=16, long_thr=thr)
    deg = np.diff(rp)
    short = deg <= thr
    assert np.array_equal(seq[short].view(np.uint32), split[short].view(np.uint32))
    assert (~short).any()
    ref, ab = O.spmm_f64(rp, ci, x, mode=O.W_GCN, dis=dis)
    assert O.check_close_to_f64(split, ref, ab) <= 1.0


def test_elementwise_oracles():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((7, 5)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    out = O.bias_relu(a, b, True)
    assert np.array_equal(out, np.maximum(a + b[None, :], np.float32(0)))
    src = rng.standard_normal((7, 5)).astype(np.float32)
    fused = O.add_inplace(a, src, 1.5)
    ref = (a.astype(np.float64) + 1.5 * src.astype(np.float64)).astype(np.float32)  # exact product, one rounding
    assert np.max(np.abs(fused - ref)) <= 1e-6 * np.max(np.abs(ref))


def test_gemm_oracle_close_to_f64():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((33, 70)).astype(np.float32)
    w = rng.standard_normal((70, 19)).astype(np.float32)
    b = rng.standard_normal(19).astype(np.float32)
    got = O.gemm_fp32(x, w, b, True)
    ref = O.gemm_f64(x, w, b, True)
    scale = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64) + np.abs(b)[None, :]
    assert np.all(np.abs(got - ref) <= 1e-5 * scale + 1e-30)


def test_split_rule_segments_and_chunks():
    """split_warps > 0: long rows are cut into segments of split_warps*512 entries,
    each cut into split_warps chunks; partials added chunk by chunk, then segment by segment."""
    from oracle import oracle as O
    rng = np.random.default_rng(5)
    n, f, deg = 6000, 3, 5000
    cols = np.sort(rng.choice(n, size=deg, replace=False)).astype(np.int32)
    rp = np.array([0, deg] + [deg] * (n - 1), dtype=np.int32)
    x = rng.standard_normal((n, f)).astype(np.float32)
    for warps in (4, 16):
        got = O.spmm(rp, cols, x, mode=O.W_UNIT, split_warps=warps, long_thr=100)[0]
        seg_len = warps * 512
        acc = None
        for sb in range(0, deg, seg_len):
            se = min(sb + seg_len, deg)
            chunk = -(-(se - sb) // warps)
            seg = None
            for w in range(warps):
                wb = min(sb + w * chunk, se)
                we = min(wb + chunk, se)
                part = np.zeros(f, dtype=np.float32)
                for e in range(wb, we):
                    part = (part + x[cols[e]]).astype(np.float32)
                seg = part if seg is None else (seg + part).astype(np.float32)
            acc = seg if acc is None else (acc + seg).astype(np.float32)
        assert np.array_equal(got.view(np.uint32), acc.view(np.uint32)), warps
        plain = O.spmm(rp, cols, x, mode=O.W_UNIT)[0]
        assert not np.array_equal(plain.view(np.uint32), got.view(np.uint32)) or warps == 0


@pytest.mark.parametrize("mode,mean", [(O.W_GCN, O.M_NONE), (O.W_EDGE, O.M_NONE), (O.W_UNIT, O.M_DIV),
                                       (O.W_UNIT, O.M_RCP)])
def test_listed_rows_equal_whole_graph_rows(graph, mode, mean):
    """spmm_rows / spmm_f64_rows on a row list, and the compact sub-problem of
    sampled rows, reproduce the whole-graph results of those rows exactly."""
    rp, ci, dis, ew, x = graph
    rows = np.array([599, 0, 17, 17, 300, 42], dtype=np.int64)
    kw = dict(mode=mode, dis=dis if mode == O.W_GCN else None, ew=ew if mode == O.W_EDGE else None, mean=mean)
    whole = O.spmm(rp, ci, x, split_warps=16, long_thr=10, **kw)
    listed = O.spmm_rows(rp, ci, x, rows, split_warps=16, long_thr=10, **kw)
    assert np.array_equal(whole[rows].view(np.uint32), listed.view(np.uint32))
    f64, ab = O.spmm_f64(rp, ci, x, **kw)
    g64, gab = O.spmm_f64_rows(rp, ci, x, rows, **kw)
    assert np.array_equal(f64[rows], g64) and np.array_equal(ab[rows], gab)
    if mode == O.W_EDGE:
        return  # the compact sub-problem carries row scales (dis), not per-entry weights
    srp, sci, sx, sdis = O.compact_rows_problem(torch.from_numpy(rp), torch.from_numpy(ci), torch.from_numpy(x),
                                                rows, torch.from_numpy(dis) if mode == O.W_GCN else None)
    k = rows.size
    sub = O.spmm(srp, sci, sx, mode=mode, dis=sdis, mean=mean, split_warps=16, long_thr=10, rows=(0, k))
    assert np.array_equal(whole[rows].view(np.uint32), sub.view(np.uint32))
    s64, sab = O.spmm_f64_rows(srp, sci, sx, np.arange(k), mode=mode, dis=sdis, mean=mean)
    assert np.allclose(s64, f64[rows], rtol=0, atol=0) and np.allclose(sab, ab[rows], rtol=0, atol=0)
