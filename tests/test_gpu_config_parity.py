"""Parity at the benchmark configurations' own sizes (run with -m gpu).

The other GPU tests use graphs of a few thousand nodes. These run the
aggregation at full size and check it against the oracle:

  * the Pubmed-shaped GCN layer (Chung-Lu, exponent 2.1, max degree ~170;
    19,717 nodes, 88,648 directed entries + 19,717 self-loops, F = 128) on
    the whole graph: bit for bit against the oracle and against the
    reference's own plain GCN kernel (gcn_ops.cu:34-109, compiled from source
    into oracle/_ref/), within 1e-5 of float64, and the layer with its TF32
    transform within 2e-3;
  * the ogbn-products-shaped GCN aggregation (2,449,029 nodes, 64,308,169
    entries) on sampled rows: every row above the long-row threshold and
    4,000 others; every sampled row bit for bit against the oracle's
    restatement of this engine's schedule; rows below the threshold also bit
    for bit against the reference kernel, long rows (summed in segments and
    chunks instead of one CSR-order chain) within 1e-5 of float64;
  * the Reddit-shaped mean aggregation (232,965 nodes, 114,615,892 entries,
    F = 256) on sampled rows, the same way, against the reference's
    csr_agg_kernel<mean> (agg_ops.cu:23-47);
  * a graph whose feature matrix has more than 2^31 elements (17,000,000 x
    128): rows with the highest ids (output offsets past 2^31) and rows that
    read columns whose feature offsets are past 2^31, for GCN and sum. The
    reference indexes these with 32-bit products (gcn_ops.cu:29,
    agg_ops.cu:38), so there the oracle alone is the check.

Tolerances: bit-exact where the order of operations is fixed (all sampled
rows against the oracle); |ours - f64| <= 1e-5 * (sum |w x| + |f64|) per
element for the fp32 aggregation; the TF32 transform within 2e-3 of
sum |a w| per element.
"""
import importlib.machinery
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200 import _native as N
from gnn_cuda_b200 import synth
from gnn_cuda_b200.GNN_cuda_common import agg_ops, gcn_ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


def _ref_module(name: str):
    """The reference's own compiled extension, or None when it was not built."""
    path = REF / f"{name}.so"
    if not path.exists():
        return None
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def _auto_long_threshold(nnz: int) -> int:
    """The engine's automatic long-row threshold: clamp(nnz / (SMs * 32 * 8), 256, 8192)."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    return max(32, min(8192, max(256, nnz // (sms * 32 * 8))))


def _bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _sample_rows(row_ptr: torch.Tensor, thr: int, n_short: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """(all long rows, n_short random other rows incl. the first and last ids)."""
    deg = (row_ptr[1:] - row_ptr[:-1]).to(torch.int64)
    long_rows = torch.nonzero(deg > thr).flatten().cpu().numpy()
    short = torch.nonzero(deg <= thr).flatten()
    g = torch.Generator(device=short.device).manual_seed(seed)
    pick = short[torch.randperm(short.numel(), generator=g, device=short.device)[:n_short]].cpu().numpy()
    n = deg.numel()
    extra = np.array([r for r in (0, n - 1) if deg[r] <= thr], dtype=np.int64)
    return long_rows.astype(np.int64), np.unique(np.concatenate([pick, extra])).astype(np.int64)


def _check_sampled(rp, ci, x, out, rows_long, rows_short, *, mode, dis=None, mean=O.M_NONE, thr, ref_out=None):
    """Sampled rows of `out` against the oracle (bits), float64 (1e-5) and the reference kernel."""
    rows = np.concatenate([rows_long, rows_short])
    k = rows.size
    srp, sci, sx, sdis = O.compact_rows_problem(rp, ci, x, rows, dis)
    exp = O.spmm(srp, sci, sx, mode=mode, dis=sdis, mean=mean, split_warps=16, long_thr=thr, rows=(0, k))
    got = out[torch.as_tensor(rows, device=out.device)].cpu().numpy()
    bad = np.nonzero(~np.all(_bits(got) == _bits(exp), axis=1))[0]
    assert bad.size == 0, f"{bad.size} sampled rows differ from the oracle, e.g. row {rows[bad[0]]}"
    f64, ab = O.spmm_f64_rows(srp, sci, sx, np.arange(k), mode=mode, dis=sdis, mean=mean)
    assert O.check_close_to_f64(got, f64, ab, rel=1e-5) <= 1.0
    if ref_out is not None and rows_short.size:
        ref_rows = ref_out[torch.as_tensor(rows_short, device=out.device)].cpu().numpy()
        short_got = got[rows_long.size:]
        assert np.array_equal(_bits(short_got), _bits(ref_rows)), "short rows differ from the reference kernel"
    return k


@pytest.fixture(autouse=True)
def _auto_threshold():
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", 0)
    yield
    N.config_set("spmm.long_row_threshold", old)
    torch.cuda.empty_cache()


def test_pubmed_shape_gcn_layer_whole_graph():
    s, d, n = synth.make_graph("gcn_pubmed_like", seed=1)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    assert n == 19_717 and s.numel() == 88_648 and ci.size == 108_365
    deg = np.diff(rp)
    assert 100 <= deg.max() <= 260  # Chung-Lu capped near 170 expected neighbours (+ the self-loop)
    f = 128
    x = synth.features(n, f, seed=2).numpy()
    w = synth.glorot(f, f, seed=3).numpy()
    b = np.zeros(f, np.float32)
    t_rp, t_ci, t_dis, t_x = (torch.from_numpy(a).to(DEV) for a in (rp, ci, dis, x))
    agg = torch.full((n, f), float("nan"), device=DEV)
    gcn_ops.spmm_gcn_forward_(t_rp, t_ci, t_dis, t_x, agg)
    out = torch.empty(n, f, device=DEV)
    torch.backends.cuda.matmul.allow_tf32 = True
    agg_ops.linear_forward_(agg, torch.from_numpy(w).to(DEV), torch.from_numpy(b).to(DEV), out, False)
    torch.cuda.synchronize()
    got = agg.cpu().numpy()
    # every row is below the long-row threshold: plain CSR order everywhere
    assert deg.max() <= _auto_long_threshold(ci.size)
    assert np.array_equal(_bits(got), _bits(O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis)))
    f64, ab = O.spmm_f64(rp, ci, x, mode=O.W_GCN, dis=dis)
    assert O.check_close_to_f64(got, f64, ab, rel=1e-5) <= 1.0
    ref = _ref_module("ref_gcn_ops")
    if ref is not None:
        ref_out = torch.full((n, f), float("nan"), device=DEV)
        ref.spmm_gcn_hmm_forward_(t_rp, t_ci, t_dis, t_x, ref_out)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(got), _bits(ref_out.cpu().numpy()))
    # the layer (aggregate, then X·W + b in TF32) against float64 of the same aggregate
    exp = O.gemm_f64(got, w, b, False)
    scale = np.abs(got.astype(np.float64)) @ np.abs(w.astype(np.float64)) + 1e-30
    assert float(np.max(np.abs(out.cpu().numpy() - exp) / scale)) <= 2e-3


def test_products_shape_gcn_sampled_rows():
    s, d, n = synth.make_graph("gcn_products_like", seed=1, device=DEV)
    rp, ci, dis = synth.csr_on_device(s, d, n, add_self_loops=True)
    del s, d
    nnz = ci.numel()
    assert n == 2_449_029 and nnz == 64_308_169
    x = synth.features(n, 128, seed=2, device=DEV)
    out = torch.full((n, 128), float("nan"), device=DEV)
    gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, out)
    ref = _ref_module("ref_gcn_ops")
    ref_out = None
    if ref is not None:
        ref_out = torch.full((n, 128), float("nan"), device=DEV)
        ref.spmm_gcn_hmm_forward_(rp, ci, dis, x, ref_out)
    torch.cuda.synchronize()
    thr = _auto_long_threshold(nnz)
    rows_long, rows_short = _sample_rows(rp, thr, 4000, seed=5)
    assert rows_long.size > 1000  # the R-MAT hubs
    _check_sampled(rp, ci, x, out, rows_long, rows_short, mode=O.W_GCN, dis=dis, thr=thr, ref_out=ref_out)


@pytest.mark.parametrize("reciprocal", [False, True])
def test_reddit_shape_mean_sampled_rows(reciprocal):
    s, d, n = synth.make_graph("sage_reddit_like", seed=1, device=DEV)
    rp, ci, _ = synth.csr_on_device(s, d, n, add_self_loops=False)
    del s, d
    nnz = ci.numel()
    assert n == 232_965 and nnz == 114_615_892
    x = synth.features(n, 256, seed=2, device=DEV)
    out = torch.full((n, 256), float("nan"), device=DEV)
    agg_ops.spmm_mean_forward_(rp, ci, x, out, hmm_optimized=reciprocal)
    ref_out = None
    ref = _ref_module("ref_agg_ops")
    if ref is not None:
        ref_out = torch.full((n, 256), float("nan"), device=DEV)
        (ref.spmm_mean_hmm_forward_ if reciprocal else ref.spmm_mean_forward_)(rp, ci, x, ref_out)
    torch.cuda.synchronize()
    thr = _auto_long_threshold(nnz)
    rows_long, rows_short = _sample_rows(rp, thr, 2000, seed=6)
    _check_sampled(rp, ci, x, out, rows_long, rows_short, mode=O.W_UNIT, mean=O.M_RCP if reciprocal else O.M_DIV,
                   thr=thr, ref_out=ref_out)


@pytest.mark.parametrize("op", ["gcn", "sum"])
def test_feature_offsets_past_2_pow_31(op):
    n, f = 17_000_000, 128
    assert n * f > 2**31
    g = torch.Generator(device=DEV).manual_seed(31)
    u = torch.randint(0, n, (3 * n,), generator=g, device=DEV)
    v = torch.randint(0, n, (3 * n,), generator=g, device=DEV)
    keep = u != v
    key = torch.unique(torch.minimum(u[keep], v[keep]) * n + torch.maximum(u[keep], v[keep]))
    del u, v, keep
    s, d = synth.symmetrize(key // n, key % n)
    del key
    rp, ci, dis = synth.csr_on_device(s, d, n, add_self_loops=op == "gcn")
    del s, d
    x = synth.features(n, f, seed=32, device=DEV)
    out = torch.full((n, f), float("nan"), device=DEV)
    if op == "gcn":
        gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, out)
    else:
        agg_ops.spmm_sum_forward_(rp, ci, x, out)
    torch.cuda.synchronize()
    # rows whose output offset is past 2^31 elements, and rows reading a column whose feature offset is
    high_rows = np.arange(n - 1500, n, dtype=np.int64)
    far = torch.nonzero(ci.to(torch.int64) * f >= 2**31).flatten()
    entry_rows = torch.searchsorted(rp.to(torch.int64), far, right=True) - 1
    far_rows = torch.unique(entry_rows)
    pick = torch.randperm(far_rows.numel(), generator=g, device=DEV)[:1500]
    rows = np.unique(np.concatenate([high_rows, far_rows[pick].cpu().numpy()]))
    assert rows.size > 2500
    thr = _auto_long_threshold(ci.numel())
    _check_sampled(rp, ci, x, out, np.zeros(0, np.int64), rows, mode=O.W_GCN if op == "gcn" else O.W_UNIT,
                   dis=dis if op == "gcn" else None, thr=thr)
