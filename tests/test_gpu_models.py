"""Model drivers end to end on the GPU against the oracle composition (run with -m gpu).

With --no-tf32 the dense transform runs the FFMA kernel, whose k-order equals
the oracle's fmaf loop, and every other op is bit-exact, so the whole GCN /
GIN / GraphSAGE forward must equal the oracle bit for bit. With TF32 (the
drivers' default) the output must stay within 1e-2 of max|out| (two TF32 GEMMs
at 2e-3 each). Placements (device, UVM, HMM when the GPU supports it) and the
--ft_host_alloc reserve must not change a single bit.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200 import _native as N
from gnn_cuda_b200 import synth
from gnn_cuda_b200.GNN_cuda_common import gcn_inference, gin_inference, graphsage_inference, npz_utils

pytestmark = pytest.mark.gpu
THR = 48


@pytest.fixture(scope="module")
def graph_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("graphs")
    u, v = synth.rmat_undirected(3000, 24000, seed=41)
    s, t = synth.symmetrize(u, v)
    npz_utils.save_graph_npz(str(d / "rmat3k.npz"), s.numpy(), t.numpy(), 3000)
    return d


@pytest.fixture(autouse=True)
def _fixed_split():
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", THR)
    yield
    N.config_set("spmm.long_row_threshold", old)


def _argv(graph_dir, *extra):
    return ["--dataset", "rmat3k", "--data_root", str(graph_dir), "--dim", "64", "--num_layers", "2",
            "--warmup", "1", "--iters", "2", "--seed", "5", *extra]


def _gcn(graph_dir, *extra, label="pyg"):
    cap = {}
    loader = npz_utils.load_pyg_graph_features_from_npz if label == "pyg" else npz_utils.load_dgl_graph_features_from_npz
    rc = gcn_inference.run_gcn_inference(framework_label=label, select_device=npz_utils.select_device,
                                         load_graph_features=loader, load_kind=label,
                                         argv=_argv(graph_dir, *extra), capture=cap)
    assert rc == 0
    return cap


def _np(t):
    return t.detach().cpu().numpy()


def _gcn_oracle(cap, *, tf32: bool):
    rp, ci = _np(cap["row_ptr"]), _np(cap["col_ind"])
    dis = O.deg_inv_sqrt_from_row_ptr(rp)
    x = _np(cap["features"])
    L = len(cap["layers"])
    for li, layer in enumerate(cap["layers"]):
        agg = O.spmm(rp, ci, x, mode=O.W_GCN, dis=dis, split_warps=16, long_thr=THR)
        w, b = _np(layer.weight), _np(layer.bias)
        x = O.gemm_f64(agg, w, b, li != L - 1).astype(np.float32) if tf32 else O.gemm_fp32(agg, w, b, li != L - 1)
    return x


def _close(got, ref, rel):
    return float(np.max(np.abs(got.astype(np.float64) - ref))) <= rel * float(np.max(np.abs(ref)) + 1e-30)


def test_gcn_fp32_bit_exact_and_placements(graph_dir, capsys):
    dev = _gcn(graph_dir, "--memory_mode", "device", "--no-tf32")
    exp = _gcn_oracle(dev, tf32=False)
    assert np.array_equal(_np(dev["output"]).view(np.uint32), exp.view(np.uint32))
    out = capsys.readouterr().out
    for line in ("Impl:\tpyg_gcn_cuda", "SpMM Kernel:\tplain_shared", "Output Sum:\t", "Summary Report:", "iter_2, "):
        assert line in out
    uvm = _gcn(graph_dir, "--memory_mode", "uvm", "--prefetch_to", "cuda", "--no-tf32")
    assert np.array_equal(_np(uvm["output"]).view(np.uint32), exp.view(np.uint32))
    out = capsys.readouterr().out
    assert "type=managed managed=True" in out
    naive = _gcn(graph_dir, "--memory_mode", "device", "--no-tf32", "--spmm_mode", "naive")
    assert np.array_equal(_np(naive["output"]).view(np.uint32), exp.view(np.uint32))
    pyg = _gcn(graph_dir, "--memory_mode", "device", "--no-tf32", "--gcn_kernel_impl", "pyg_baseline")
    assert np.array_equal(_np(pyg["output"]).view(np.uint32), exp.view(np.uint32))


def test_gcn_tf32_default(graph_dir):
    cap = _gcn(graph_dir, "--memory_mode", "device")
    assert _close(_np(cap["output"]), _gcn_oracle(cap, tf32=True), 1e-2)


def test_gcn_ft_host_alloc_reserve(graph_dir, capsys):
    ref = _gcn(graph_dir, "--memory_mode", "device", "--no-tf32")
    capsys.readouterr()
    cap = _gcn(graph_dir, "--adj_matrix", "device", "--weight", "device", "--ft_matrix", "uvm", "--ft_host_alloc", "20",
               "--prefetch_to", "cuda", "--no-tf32")
    out = capsys.readouterr().out
    assert "Feature Reserve Enabled:\tTrue" in out
    act = [l for l in out.splitlines() if l.startswith("Reserve Activations:")]
    assert act and int(act[0].split("\t")[1]) >= 3  # setup + warmup + 2 iters
    assert "Feature Preferred Location:\tcpu" in out
    assert np.array_equal(_np(cap["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))


def test_gcn_optimized_mode_with_metadata(graph_dir, tmp_path, capsys):
    n = 3000
    meta = {"row_schedule": torch.arange(n - 1, -1, -1, dtype=torch.long), "hot_node_cutoff": 256,
            "hot_node_fraction": 256 / n, "rows_per_page": 8}
    path = tmp_path / "meta.pt"
    torch.save(meta, path)
    ref = _gcn(graph_dir, "--memory_mode", "device", "--no-tf32")
    capsys.readouterr()
    cap = _gcn(graph_dir, "--adj_matrix", "device", "--weight", "device", "--ft_matrix", "uvm", "--spmm_mode",
               "optimized", "--preprocess_meta", str(path), "--no-tf32")
    out = capsys.readouterr().out
    assert "Optimized Managed Active:\tTrue" in out and "SpMM Kernel:\toptimized_uvm" in out
    assert np.array_equal(_np(cap["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))


def test_gcn_hmm_placement(graph_dir):
    import ctypes
    ok = ctypes.c_int(0)
    N.check(N.lib().gnn_hmm_supported(0, ctypes.byref(ok)))
    if not ok.value:
        pytest.skip("this GPU/driver does not report pageable memory access (HMM)")
    ref = _gcn(graph_dir, "--memory_mode", "device", "--no-tf32")
    cap = _gcn(graph_dir, "--adj_matrix", "hmm", "--ft_matrix", "hmm", "--weight", "device", "--no-tf32")
    assert np.array_equal(_np(cap["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))


def _gin(graph_dir, post, *extra):
    cap = {}
    rc = gin_inference.run_gin_inference(framework_label="dgl" if post else "pyg", select_device=npz_utils.select_device,
                                         load_graph_features=npz_utils.load_dgl_graph_features_from_npz,
                                         load_kind="dgl", post_layer_relu=post, argv=_argv(graph_dir, *extra),
                                         capture=cap)
    assert rc == 0
    return cap


def _sage(graph_dir, *extra):
    cap = {}
    rc = graphsage_inference.run_graphsage_inference(
        framework_label="pyg", select_device=npz_utils.select_device,
        load_graph_features=npz_utils.load_pyg_graph_features_from_npz, load_kind="pyg",
        argv=_argv(graph_dir, *extra), capture=cap)
    assert rc == 0
    return cap


@pytest.mark.parametrize("post", [False, True])
def test_gin_fp32_bit_exact(graph_dir, post):
    cap = _gin(graph_dir, post, "--memory_mode", "device", "--no-tf32")
    rp, ci = _np(cap["row_ptr"]), _np(cap["col_ind"])
    x = _np(cap["features"])
    L = len(cap["layers"])
    for li, layer in enumerate(cap["layers"]):
        agg = O.spmm(rp, ci, x, mode=O.W_UNIT, split_warps=16, long_thr=THR)
        agg = O.add_inplace(agg, x, np.float32(layer.alpha))
        hid = O.gemm_fp32(agg, _np(layer.weight1), _np(layer.bias1), True)
        x = O.gemm_fp32(hid, _np(layer.weight2), _np(layer.bias2), post and li != L - 1)
    assert np.array_equal(_np(cap["output"]).view(np.uint32), x.view(np.uint32))
    uvm = _gin(graph_dir, post, "--memory_mode", "uvm", "--no-tf32")
    assert np.array_equal(_np(uvm["output"]).view(np.uint32), x.view(np.uint32))


def test_graphsage_fp32_bit_exact(graph_dir):
    cap = {}
    rc = graphsage_inference.run_graphsage_inference(
        framework_label="pyg", select_device=npz_utils.select_device,
        load_graph_features=npz_utils.load_pyg_graph_features_from_npz, load_kind="pyg",
        argv=_argv(graph_dir, "--memory_mode", "device", "--no-tf32"), capture=cap)
    assert rc == 0
    rp, ci = _np(cap["row_ptr"]), _np(cap["col_ind"])
    x = _np(cap["features"])
    L = len(cap["layers"])
    for li, layer in enumerate(cap["layers"]):
        agg = O.spmm(rp, ci, x, mode=O.W_UNIT, mean=O.M_DIV, split_warps=16, long_thr=THR)
        out = O.gemm_fp32(agg, _np(layer.weight_neigh), _np(layer.bias_neigh), False)
        root = O.gemm_fp32(x, _np(layer.weight_root), None, False)
        out = O.add_inplace(out, root, np.float32(1.0))
        x = O.relu(out) if li != L - 1 else out
    assert np.array_equal(_np(cap["output"]).view(np.uint32), x.view(np.uint32))


def test_fused_layers_equal_separate_calls_in_every_driver(graph_dir):
    """--fuse_layers (one kernel per layer, no aggregate buffer) returns the same bits
    as the separate calls on the TF32 path, for GCN, GIN and GraphSAGE-mean."""
    ref, fused = _gcn(graph_dir), _gcn(graph_dir, "--fuse_layers")
    assert np.array_equal(_np(fused["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))
    assert all(layer.agg_buffer.numel() == 0 for layer in fused["layers"])
    for post in (False, True):
        ref, fused = _gin(graph_dir, post), _gin(graph_dir, post, "--fuse_layers")
        assert np.array_equal(_np(fused["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))
    ref, fused = _sage(graph_dir), _sage(graph_dir, "--fuse_layers")
    assert np.array_equal(_np(fused["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))


def test_transform_first_order_within_tf32_tolerance(graph_dir):
    """--layer_order transform_first computes A·(x·W): the same layer up to the
    rounding of a different association, held to the TF32 tolerance of the oracle."""
    cap = _gcn(graph_dir, "--layer_order", "transform_first")
    assert _close(_np(cap["output"]), _gcn_oracle(cap, tf32=True), 1e-2)
    ref = _gin(graph_dir, True)
    got = _gin(graph_dir, True, "--layer_order", "transform_first")
    assert _close(_np(got["output"]), _np(ref["output"]).astype(np.float64), 1e-2)
    ref = _sage(graph_dir)
    got = _sage(graph_dir, "--layer_order", "transform_first")
    assert _close(_np(got["output"]), _np(ref["output"]).astype(np.float64), 1e-2)


def test_overlapped_prefetch_same_bits(graph_dir):
    """--prefetch_pieces: unified-memory features prefetched in row ranges on a side
    stream during the forward, the first aggregation in row pieces that wait only
    for their range — the same output bits as the prefetch before the loop."""
    base = ("--ft_matrix", "uvm", "--prefetch_to", "cuda", "--preferred_location", "cuda")
    ref = _gcn(graph_dir, *base)
    got = _gcn(graph_dir, *base, "--prefetch_pieces", "4")
    assert np.array_equal(_np(got["output"]).view(np.uint32), _np(ref["output"]).view(np.uint32))
