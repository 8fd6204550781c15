"""Pin the oracle (and this package) against the reference's own CUDA kernels.

oracle/build_ref.py compiles the reference's gcn_ops / pyg_gcn_ops / agg_ops
extensions from their sources into oracle/_ref/. On a B200 this test runs the
reference kernels on the same seeded tensors and checks, bit for bit, that
  reference kernel == C oracle == libgnnb200
for every row that libgnnb200 accumulates in plain CSR order (all rows when
the long-row split is disabled by a huge threshold). The reference's naive
kernels index with 32-bit `col * feat_dim` (gcn_ops.cu:29, agg_ops.cu:38), so
the sizes here stay far below 2^31 elements.
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
from gnn_cuda_b200.GNN_cuda_common import agg_ops, gcn_ops, pyg_gcn_ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


def _load(name: str):
    path = REF / f"{name}.so"
    if not path.exists():
        pytest.skip(f"{path} not built (python oracle/build_ref.py)")
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def ref():
    return {n: _load(n) for n in ("ref_gcn_ops", "ref_pyg_gcn_ops", "ref_agg_ops")}


@pytest.fixture(autouse=True)
def _no_split():
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", 1 << 40)  # every row in plain CSR order
    yield
    N.config_set("spmm.long_row_threshold", old)


def _bits(t):
    return t.detach().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("f", [3, 128, 129, 256])
def test_gcn_three_way_bit_exact(ref, f):
    n = 4000
    u, v = synth.rmat_undirected(n, n * 10, seed=21)
    s, d = synth.symmetrize(u, v)
    rp, ci, dis = O.gcn_normalized_csr(s.numpy(), d.numpy(), n)
    _, _, ew = O.pyg_weighted_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=22).numpy()
    oracle_out = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis)
    t_rp, t_ci, t_dis, t_ew, t_x = (torch.from_numpy(a).to(DEV) for a in (rp, ci, dis, ew, x))
    outs = {}
    for name, fn in (("ref_naive", ref["ref_gcn_ops"].spmm_gcn_forward_),
                     ("ref_plain", ref["ref_gcn_ops"].spmm_gcn_hmm_forward_)):
        o = torch.full((n, f), float("nan"), device=DEV)
        fn(t_rp, t_ci, t_dis, t_x, o)
        outs[name] = o
    for name, fn in (("ref_pyg_naive", ref["ref_pyg_gcn_ops"].spmm_pyg_gcn_forward_),
                     ("ref_pyg_plain", ref["ref_pyg_gcn_ops"].spmm_pyg_gcn_plain_forward_)):
        o = torch.full((n, f), float("nan"), device=DEV)
        fn(t_rp, t_ci, t_ew, t_x, o)
        outs[name] = o
    mine = torch.empty(n, f, device=DEV)
    gcn_ops.spmm_gcn_forward_(t_rp, t_ci, t_dis, t_x, mine)
    mine_pyg = torch.empty(n, f, device=DEV)
    pyg_gcn_ops.spmm_pyg_gcn_forward_(t_rp, t_ci, t_ew, t_x, mine_pyg)
    torch.cuda.synchronize()
    for name, o in outs.items():
        assert np.array_equal(_bits(o), oracle_out.view(np.uint32)), f"oracle != {name}"
    assert np.array_equal(_bits(mine), oracle_out.view(np.uint32))
    assert np.array_equal(_bits(mine_pyg), oracle_out.view(np.uint32))


@pytest.mark.parametrize("f", [5, 128, 256])
def test_sum_mean_three_way_bit_exact(ref, f):
    n = 3000
    u, v = synth.community_lognormal(n, n * 20, seed=31)
    s, d = synth.symmetrize(u, v)
    rp, ci = O.plain_csr(s.numpy(), d.numpy(), n)
    x = synth.features(n, f, seed=32).numpy()
    t_rp, t_ci, t_x = (torch.from_numpy(a).to(DEV) for a in (rp, ci, x))
    A = ref["ref_agg_ops"]
    cases = [(A.spmm_sum_forward_, O.M_NONE, agg_ops.spmm_sum_forward_, False),
             (A.spmm_sum_hmm_forward_, O.M_NONE, agg_ops.spmm_sum_forward_, True),
             (A.spmm_mean_forward_, O.M_DIV, agg_ops.spmm_mean_forward_, False),
             (A.spmm_mean_hmm_forward_, O.M_RCP, agg_ops.spmm_mean_forward_, True)]
    for ref_fn, mean, my_fn, hmm in cases:
        exp = O.spmm(rp, ci, x, mode=O.W_UNIT, mean=mean)
        o = torch.full((n, f), float("nan"), device=DEV)
        ref_fn(t_rp, t_ci, t_x, o)
        mine = torch.empty(n, f, device=DEV)
        my_fn(t_rp, t_ci, t_x, mine, hmm_optimized=hmm)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(o), exp.view(np.uint32)), (ref_fn.__name__, "oracle")
        assert np.array_equal(_bits(mine), exp.view(np.uint32)), (ref_fn.__name__, "mine")


def test_elementwise_three_way(ref):
    A = ref["ref_agg_ops"]
    g = torch.Generator().manual_seed(5)
    a = torch.randn(300, 40, generator=g)
    b = torch.randn(40, generator=g)
    src = torch.randn(300, 40, generator=g)
    r1, m1 = a.to(DEV), a.to(DEV)
    A.bias_relu_forward_(r1, b.to(DEV), True)
    agg_ops.bias_relu_forward_(m1, b.to(DEV), True)
    A.tensor_add_inplace_(r1, src.to(DEV), 1.25)
    agg_ops.tensor_add_inplace_(m1, src.to(DEV), 1.25)
    A.relu_inplace_(r1)
    agg_ops.relu_inplace_(m1)
    exp = O.relu(O.add_inplace(O.bias_relu(a.numpy(), b.numpy(), True), src.numpy(), np.float32(1.25)))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(r1), exp.view(np.uint32))
    assert np.array_equal(_bits(m1), exp.view(np.uint32))


def test_reference_sgemm_vs_ours(ref):
    """cublasSgemm (the reference's GEMM) and our FP32 / TF32 kernels against float64."""
    A = ref["ref_agg_ops"]
    g = torch.Generator().manual_seed(6)
    x = torch.randn(2048, 128, generator=g)
    w = torch.randn(128, 128, generator=g)
    scale = np.abs(x.numpy()).astype(np.float64) @ np.abs(w.numpy()).astype(np.float64)
    ref64 = O.gemm_f64(x.numpy(), w.numpy())
    r = torch.empty(2048, 128, device=DEV)
    A.gemm_forward_(x.to(DEV), w.to(DEV), r)
    for precision, tol in ((N.GNN_PRECISION_FP32, 1e-5), (N.GNN_PRECISION_TF32, 2e-3)):
        m = torch.empty(2048, 128, device=DEV)
        from gnn_cuda_b200.GNN_cuda_common import native_ops
        native_ops.gemm_forward_(x.to(DEV), w.to(DEV), m, precision=precision)
        assert np.all(np.abs(m.cpu().numpy() - ref64) <= tol * scale)
    assert np.all(np.abs(r.cpu().numpy() - ref64) <= 1e-5 * scale)
