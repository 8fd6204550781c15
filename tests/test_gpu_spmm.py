"""GPU parity of the aggregation kernels against the C oracle (run with -m gpu).

Bit-exact checks: rows accumulated by one warp follow the reference's CSR
order, so they must equal the oracle's fmaf/add sequence bit for bit; long
rows follow the documented warp split, which the oracle reproduces with
``split_warps`` — so every output element is compared exactly. Every case is
also held to the fp32 tolerance of 1e-5 (relative to the summed magnitudes) against float64.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200 import _native as N
from gnn_cuda_b200 import synth
from gnn_cuda_b200.GNN_cuda_common import agg_ops, gcn_ops, native_ops, pyg_gcn_ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _graph(kind: str, n: int, seed: int):
    if kind == "powerlaw":
        u, v = synth.chung_lu_undirected(n, n * 6, max_degree=300.0, seed=seed)
    elif kind == "rmat":
        u, v = synth.rmat_undirected(n, n * 8, seed=seed)
    elif kind == "hub":  # one row of degree ~n, rows of degree 0, 1, 31, 32, 33
        hub = torch.arange(1, n, dtype=torch.int64)
        u = torch.cat([torch.zeros(n - 1, dtype=torch.int64), torch.full((31,), 2), torch.full((32,), 3),
                       torch.full((33,), 4), torch.tensor([5])])
        v = torch.cat([hub, torch.arange(100, 131), torch.arange(200, 232), torch.arange(300, 333), torch.tensor([7])])
        keep = u != v
        u, v = u[keep], v[keep]
        key = torch.unique(torch.minimum(u, v) * n + torch.maximum(u, v))
        u, v = key // n, key % n
    else:
        raise ValueError(kind)
    return synth.symmetrize(u, v)


@pytest.fixture(autouse=True)
def _restore_config():
    thr, warps = N.config_get("spmm.long_row_threshold"), N.config_get("spmm.long_row_warps")
    yield
    N.config_set("spmm.long_row_threshold", thr)
    N.config_set("spmm.long_row_warps", warps)


def _bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _expected(rp, ci, x, *, mode, dis=None, ew=None, mean=O.M_NONE, vector=True, thr=None, warps=16):
    split = warps if (vector and thr is not None) else 0
    return O.spmm(rp, ci, x, mode=mode, dis=dis, ew=ew, mean=mean, split_warps=split, long_thr=thr or 0)


CASES = [("powerlaw", 3000, f) for f in (1, 3, 4, 31, 64, 128, 129, 256, 512, 640)] + \
        [("rmat", 4096, 128), ("hub", 3000, 128), ("hub", 3000, 256), ("hub", 3000, 31)]


@pytest.mark.parametrize("kind,n,f", CASES)
@pytest.mark.parametrize("thr", [48, None])
def test_gcn_and_pyg_bit_exact(kind, n, f, thr):
    s, d = _graph(kind, n, seed=7)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    _, _, ew = O.pyg_weighted_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=3).numpy()
    N.config_set("spmm.long_row_threshold", thr or 0)
    eff_thr = thr if thr is not None else 256  # automatic threshold floor for graphs this small
    vector = f % 4 == 0
    exp = _expected(rp, ci, x, mode=O.W_GCN, dis=dis, vector=vector, thr=eff_thr)
    ref64, ab = O.spmm_f64(rp, ci, x, mode=O.W_GCN, dis=dis)
    t = {k: torch.from_numpy(v).to(DEV) for k, v in dict(rp=rp, ci=ci, dis=dis, ew=ew, x=x).items()}
    for mode in ("naive", "plain"):
        out = torch.full((n, f), float("nan"), device=DEV)
        gcn_ops.spmm_gcn_forward_(t["rp"], t["ci"], t["dis"], t["x"], out, spmm_mode=mode)
        got = out.cpu().numpy()
        assert _bits_equal(got, exp), (mode, np.max(np.abs(got - exp)))
        assert O.check_close_to_f64(got, ref64, ab) <= 1.0
        out2 = torch.full((n, f), float("nan"), device=DEV)
        pyg_gcn_ops.spmm_pyg_gcn_forward_(t["rp"], t["ci"], t["ew"], t["x"], out2, spmm_mode=mode)
        assert _bits_equal(out2.cpu().numpy(), exp)


@pytest.mark.parametrize("f", [4, 128, 129, 256])
@pytest.mark.parametrize("thr", [40, None])
def test_sum_and_mean_bit_exact(f, thr):
    n = 2500
    s, d = _graph("powerlaw", n, seed=9)
    rp, ci = O.plain_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=4).numpy()
    N.config_set("spmm.long_row_threshold", thr or 0)
    eff_thr = thr if thr is not None else 256
    vector = f % 4 == 0
    t_rp, t_ci, t_x = (torch.from_numpy(a).to(DEV) for a in (rp, ci, x))
    for mean, fn in ((O.M_NONE, agg_ops.spmm_sum_forward_), (O.M_DIV, agg_ops.spmm_mean_forward_)):
        for hmm in (False, True):
            m = O.M_RCP if (mean == O.M_DIV and hmm) else mean
            exp = _expected(rp, ci, x, mode=O.W_UNIT, mean=m, vector=vector, thr=eff_thr)
            out = torch.full((n, f), float("nan"), device=DEV)
            fn(t_rp, t_ci, t_x, out, hmm_optimized=hmm)
            got = out.cpu().numpy()
            assert _bits_equal(got, exp), (mean, hmm)
            ref64, ab = O.spmm_f64(rp, ci, x, mode=O.W_UNIT, mean=m)
            assert O.check_close_to_f64(got, ref64, ab) <= 1.0


def test_int64_row_ptr_and_optimized_mode():
    n, f = 3000, 128
    s, d = _graph("hub", n, seed=1)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=2).numpy()
    N.config_set("spmm.long_row_threshold", 64)
    exp = _expected(rp, ci, x, mode=O.W_GCN, dis=dis, thr=64)
    t_rp64 = torch.from_numpy(rp.astype(np.int64)).to(DEV)
    t_ci, t_dis, t_x = (torch.from_numpy(a).to(DEV) for a in (ci, dis, x))
    out = torch.empty(n, f, device=DEV)
    gcn_ops.spmm_gcn_forward_(t_rp64, t_ci, t_dis, t_x, out)
    assert _bits_equal(out.cpu().numpy(), exp)
    # optimized: reversed row schedule + a hot cache holding the first 500 rows
    sched = torch.arange(n - 1, -1, -1, dtype=torch.int64, device=DEV)
    hot = t_x[:500].clone()
    out2 = torch.empty(n, f, device=DEV)
    gcn_ops.spmm_gcn_forward_(t_rp64, t_ci, t_dis, t_x, out2, spmm_mode="optimized", row_schedule=sched,
                              hot_feature_cache=hot, hot_node_cutoff=500)
    assert _bits_equal(out2.cpu().numpy(), exp)
    # the hot cache is really read: a scaled cache changes exactly the contributions of hot columns
    hot_scaled = hot * 2.0
    out3 = torch.empty(n, f, device=DEV)
    gcn_ops.spmm_gcn_forward_(t_rp64, t_ci, t_dis, t_x, out3, spmm_mode="optimized", row_schedule=sched,
                              hot_feature_cache=hot_scaled, hot_node_cutoff=500)
    exp3 = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, hot=hot_scaled.cpu().numpy(), hot_cutoff=500, split_warps=16,
                  long_thr=64)
    assert _bits_equal(out3.cpu().numpy(), exp3)


def test_edge_cases_empty_and_single():
    # no edges: every row is 0 (mean of degree 0 is 0)
    n, f = 37, 128
    rp = torch.zeros(n + 1, dtype=torch.int32, device=DEV)
    ci = torch.zeros(0, dtype=torch.int32, device=DEV)
    x = torch.randn(n, f, device=DEV)
    out = torch.full((n, f), 7.0, device=DEV)
    agg_ops.spmm_mean_forward_(rp, ci, x, out)
    assert torch.count_nonzero(out).item() == 0
    # one node with a self-loop
    rp1 = torch.tensor([0, 1], dtype=torch.int32, device=DEV)
    ci1 = torch.tensor([0], dtype=torch.int32, device=DEV)
    x1 = torch.randn(1, 4, device=DEV)
    o1 = torch.empty(1, 4, device=DEV)
    agg_ops.spmm_sum_forward_(rp1, ci1, x1, o1)
    assert torch.equal(o1, x1)


def test_unaligned_views_take_scalar_path():
    n, f = 500, 128
    s, d = _graph("powerlaw", n, seed=5)
    rp, ci = O.plain_csr(s.numpy(), d.numpy(), n)
    base = synth.features(n * f + 1, 1, seed=8).numpy().reshape(-1)
    x = base[1:].reshape(n, f)  # 4-byte offset: not 16-byte aligned
    exp = O.spmm(rp, ci, x, mode=O.W_UNIT)
    t_base = torch.from_numpy(base).to(DEV)
    t_x = t_base[1:].view(n, f)
    out = torch.empty(n, f, device=DEV)
    agg_ops.spmm_sum_forward_(torch.from_numpy(rp).to(DEV), torch.from_numpy(ci).to(DEV), t_x, out)
    assert _bits_equal(out.cpu().numpy(), exp)


def test_mapped_host_inputs():
    """CPU tensors in pinned (mapped) memory are read through their device alias."""
    n, f = 800, 64
    s, d = _graph("powerlaw", n, seed=2)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=1).numpy()
    exp = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis)
    pin = [torch.from_numpy(a).pin_memory() for a in (rp, ci, dis, x)]
    out = torch.empty(n, f, device=DEV)
    gcn_ops.spmm_gcn_forward_(*pin, out)
    torch.cuda.synchronize()
    assert _bits_equal(out.cpu().numpy(), exp)


def test_stage_kernels():
    x = torch.randn(100, 12, device=DEV)
    out = torch.empty(30, 12, device=DEV)
    gcn_ops.stage_feature_rows_(x, out)
    assert torch.equal(out, x[:30])
    pages = torch.tensor([3, 0, 24], dtype=torch.int64, device=DEV)
    po = torch.empty(12, 12, device=DEV)
    gcn_ops.stage_feature_pages_(pages, x, po, rows_per_page=4)
    exp = torch.zeros(12, 12, device=DEV)
    for i, p in enumerate([3, 0, 24]):
        for j in range(4):
            node = p * 4 + j
            if node < 100:
                exp[i * 4 + j] = x[node]
    assert torch.equal(po, exp)


def test_workspace_reuse_and_streams():
    """Two back-to-back calls on a side stream reuse one workspace and stay exact."""
    n, f = 4000, 128
    s, d = _graph("rmat", n, seed=4)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=9).numpy()
    N.config_set("spmm.long_row_threshold", 32)
    exp = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=16, long_thr=32)
    t = [torch.from_numpy(a).to(DEV) for a in (rp, ci, dis, x)]
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        o1 = torch.empty(n, f, device=DEV)
        o2 = torch.empty(n, f, device=DEV)
        gcn_ops.spmm_gcn_forward_(*t, o1)
        gcn_ops.spmm_gcn_forward_(*t, o2)
    side.synchronize()
    assert _bits_equal(o1.cpu().numpy(), exp) and _bits_equal(o2.cpu().numpy(), exp)
    assert len(native_ops._workspaces) >= 1


@pytest.mark.parametrize("f", [128, 256, 512, 640])
def test_stream_and_per_row_kernels_identical(f):
    """The packed-stream kernel (default) and the one-warp-per-row kernel give the same bits."""
    n = 5000
    s, d = _graph("rmat", n, seed=12)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=13).numpy()
    t = [torch.from_numpy(a).to(DEV) for a in (rp, ci, dis, x)]
    outs = []
    old = N.config_get("spmm.kernel")
    try:
        for kern in (0, 1, 2):
            N.config_set("spmm.kernel", kern)
            o = torch.full((n, f), float("nan"), device=DEV)
            gcn_ops.spmm_gcn_forward_(*t, o)
            outs.append(o.cpu().numpy())
    finally:
        N.config_set("spmm.kernel", old)
    assert _bits_equal(outs[0], outs[1]) and _bits_equal(outs[0], outs[2])
    exp = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=16, long_thr=256)
    assert _bits_equal(outs[0], exp)


@pytest.mark.parametrize("kern", [1, 2])
@pytest.mark.parametrize("f", [4, 128, 256])
def test_alternative_kernels_all_modes(kern, f):
    """Kernels 1 and 2 against the oracle for every weight/mean mode, with long rows."""
    n = 3000
    s, d = _graph("hub", n, seed=14)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    _, _, ew = O.pyg_weighted_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=15).numpy()
    t = {k: torch.from_numpy(v).to(DEV) for k, v in dict(rp=rp, ci=ci, dis=dis, ew=ew, x=x).items()}
    old = N.config_get("spmm.kernel")
    N.config_set("spmm.kernel", kern)
    N.config_set("spmm.long_row_threshold", 40)
    try:
        cases = [(lambda o: gcn_ops.spmm_gcn_forward_(t["rp"], t["ci"], t["dis"], t["x"], o),
                  dict(mode=O.W_GCN, dis=dis)),
                 (lambda o: pyg_gcn_ops.spmm_pyg_gcn_forward_(t["rp"], t["ci"], t["ew"], t["x"], o),
                  dict(mode=O.W_EDGE, ew=ew)),
                 (lambda o: agg_ops.spmm_sum_forward_(t["rp"], t["ci"], t["x"], o), dict(mode=O.W_UNIT)),
                 (lambda o: agg_ops.spmm_mean_forward_(t["rp"], t["ci"], t["x"], o),
                  dict(mode=O.W_UNIT, mean=O.M_DIV)),
                 (lambda o: agg_ops.spmm_mean_forward_(t["rp"], t["ci"], t["x"], o, hmm_optimized=True),
                  dict(mode=O.W_UNIT, mean=O.M_RCP))]
        for run, kw in cases:
            o = torch.full((n, f), float("nan"), device=DEV)
            run(o)
            exp = O.spmm(rp, ci, x, split_warps=16, long_thr=40, **kw)
            assert _bits_equal(o.cpu().numpy(), exp), kw
    finally:
        N.config_set("spmm.kernel", old)


def test_long_row_warp_counts():
    n, f = 3000, 128
    s, d = _graph("hub", n, seed=3)
    rp, ci = O.plain_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=6).numpy()
    t = [torch.from_numpy(a).to(DEV) for a in (rp, ci, x)]
    for warps in (4, 8, 16):
        N.config_set("spmm.long_row_warps", warps)
        N.config_set("spmm.long_row_threshold", 100)
        exp = O.spmm(rp, ci, x, mode=O.W_UNIT, split_warps=warps, long_thr=100)
        out = torch.empty(n, f, device=DEV)
        agg_ops.spmm_sum_forward_(*t, out)
        assert _bits_equal(out.cpu().numpy(), exp), warps


def _hub_graph(n: int, hub_degrees, extra: int, seed: int):
    """Rows 0..len(hub_degrees)-1 are hubs of about the given degrees, plus random pairs."""
    rng = np.random.default_rng(seed)
    us, vs = [], []
    for h, deg in enumerate(hub_degrees):
        cols = rng.choice(np.arange(len(hub_degrees), n), size=deg, replace=False)
        us.append(np.full(deg, h))
        vs.append(cols)
    us.append(rng.integers(0, n, extra))
    vs.append(rng.integers(0, n, extra))
    u = torch.from_numpy(np.concatenate(us).astype(np.int64))
    v = torch.from_numpy(np.concatenate(vs).astype(np.int64))
    keep = u != v
    u, v = u[keep], v[keep]
    key = torch.unique(torch.minimum(u, v) * n + torch.maximum(u, v))
    return synth.symmetrize(key // n, key % n)


@pytest.mark.parametrize("f", [128, 640])
def test_multi_segment_hubs_all_kernels(f):
    """Rows longer than one segment (warps x 512 entries) are summed by several CTAs
    chained in segment order; every kernel and weight mode matches the oracle bit for bit."""
    n = 120_000
    s, d = _hub_graph(n, [100_001, 50_000, 20_000, 9_000, 8_193, 8_192], extra=150_000, seed=21)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    _, _, ew = O.pyg_weighted_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=22).numpy()
    assert np.diff(rp).max() > 100_000
    t = {k: torch.from_numpy(v).to(DEV) for k, v in dict(rp=rp, ci=ci, dis=dis, ew=ew, x=x).items()}
    old = N.config_get("spmm.kernel")
    try:
        for warps in (16, 4):
            N.config_set("spmm.long_row_warps", warps)
            N.config_set("spmm.long_row_threshold", 300)
            exp_gcn = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=warps, long_thr=300)
            exp_mean = O.spmm(rp, ci, x, mode=O.W_UNIT, mean=O.M_DIV, split_warps=warps, long_thr=300)
            for kern in (1, 0, 2):
                N.config_set("spmm.kernel", kern)
                o = torch.full((n, f), float("nan"), device=DEV)
                gcn_ops.spmm_gcn_forward_(t["rp"], t["ci"], t["dis"], t["x"], o)
                assert _bits_equal(o.cpu().numpy(), exp_gcn), (warps, kern, "gcn")
                o2 = torch.full((n, f), float("nan"), device=DEV)
                agg_ops.spmm_mean_forward_(t["rp"], t["ci"], t["x"], o2)
                assert _bits_equal(o2.cpu().numpy(), exp_mean), (warps, kern, "mean")
        ref64, ab = O.spmm_f64(rp, ci, x, mode=O.W_GCN, dis=dis)
        assert O.check_close_to_f64(exp_gcn, ref64, ab) <= 1.0
    finally:
        N.config_set("spmm.kernel", old)
    status = ctypes.c_int(-1)  # no segment gave up waiting for its predecessor
    N.check(N.lib().gnn_device_status(1, ctypes.byref(status)))
    assert status.value == 0


@pytest.mark.parametrize("idx", [torch.int32, torch.int64])
def test_degree_schedule_matches_row_order_and_oracle(idx):
    """With the schedule-sized workspace the per-row kernel takes rows in descending
    degree order (counting sort per call); with the minimum workspace it takes
    them in id order. Both must equal the oracle bit for bit (each row is still
    summed alone in CSR order), for every weight mode, on a graph large enough
    (>= 65,536 rows) for the schedule to be built."""
    n, f = 150_000, 128
    s, d = _graph("rmat", n, seed=31)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=32).numpy()
    t = {k: torch.from_numpy(v).to(DEV) for k, v in dict(rp=rp, ci=ci, dis=dis, x=x).items()}
    t["rp"] = t["rp"].to(idx)
    L = N.lib()
    nnz = int(ci.size)
    small = int(L.gnn_spmm_workspace_bytes(n, nnz))
    big = int(L.gnn_spmm_schedule_workspace_bytes(n, nnz))
    assert big > small + n * 4 - 1
    it = N.GNN_INDEX_INT64 if idx == torch.int64 else N.GNN_INDEX_INT32
    stream = torch.cuda.current_stream(DEV).cuda_stream
    keys = ("spmm.kernel", "spmm.long_row_threshold", "spmm.long_row_warps", "spmm.schedule", "spmm.schedule_window")
    old = [N.config_get(k) for k in keys]
    N.config_set("spmm.kernel", 1)
    N.config_set("spmm.long_row_threshold", 256)
    N.config_set("spmm.long_row_warps", 16)
    try:
        for mode, exp in (("gcn", O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=16, long_thr=256)),
                          ("sum", O.spmm(rp, ci, x, mode=O.W_UNIT, split_warps=16, long_thr=256))):
            outs = []
            runs = [(small, 1, 4096), (big, 0, 4096), (big, 1, 4096), (big, 1, 1024), (big, 1, 1 << 20), (big, 2, 4096)]
            for nbytes, sched, window in runs:
                N.config_set("spmm.schedule", sched)
                N.config_set("spmm.schedule_window", window)
                ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
                o = torch.full((n, f), float("nan"), device=DEV)
                if mode == "gcn":
                    rc = L.gnn_spmm_gcn_forward(t["rp"].data_ptr(), it, t["ci"].data_ptr(), t["dis"].data_ptr(),
                                                t["x"].data_ptr(), o.data_ptr(), n, nnz, f, ws.data_ptr(), nbytes,
                                                ctypes.c_void_p(stream))
                else:
                    rc = L.gnn_spmm_sum_forward(t["rp"].data_ptr(), it, t["ci"].data_ptr(), t["x"].data_ptr(),
                                                o.data_ptr(), n, nnz, f, ws.data_ptr(), nbytes,
                                                ctypes.c_void_p(stream))
                N.check(rc)
                outs.append(o.cpu().numpy())
            for o, run in zip(outs, runs):
                assert _bits_equal(o, exp), (mode, run)
    finally:
        for k, v in zip(keys, old):
            N.config_set(k, v)


@pytest.mark.parametrize("f", [128, 256])
def test_dense_graph_two_rows_per_warp(f):
    """Graphs with 64 or more entries per row on average take the per-row kernel
    with two rows per warp and the windowed degree order: still bit-exact."""
    n = 70_000
    u, v = synth.community_lognormal(n, n * 40, seed=41)
    s, d = synth.symmetrize(u, v)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    assert ci.size >= 64 * n
    x = synth.features(n, f, seed=42).numpy()
    t = {k: torch.from_numpy(a).to(DEV) for k, a in dict(rp=rp, ci=ci, dis=dis, x=x).items()}
    keys = ("spmm.kernel", "spmm.long_row_threshold", "spmm.long_row_warps", "spmm.schedule")
    old = [N.config_get(k) for k in keys]
    for k, v in zip(keys, (1, 1024, 16, 3)):
        N.config_set(k, v)
    try:
        exp_gcn = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=16, long_thr=1024)
        exp_mean = O.spmm(rp, ci, x, mode=O.W_UNIT, mean=O.M_DIV, split_warps=16, long_thr=1024)
        o = torch.full((n, f), float("nan"), device=DEV)
        gcn_ops.spmm_gcn_forward_(t["rp"], t["ci"], t["dis"], t["x"], o)
        assert _bits_equal(o.cpu().numpy(), exp_gcn)
        o2 = torch.full((n, f), float("nan"), device=DEV)
        agg_ops.spmm_mean_forward_(t["rp"], t["ci"], t["x"], o2)
        assert _bits_equal(o2.cpu().numpy(), exp_mean)
    finally:
        for k, v in zip(keys, old):
            N.config_set(k, v)
