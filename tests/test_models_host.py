"""Model drivers on the host: flag surface and error behaviour (no GPU needed)."""
import pytest
import torch

from gnn_cuda_b200.GNN_cuda_common import gcn_inference, gin_inference, graphsage_inference
from gnn_cuda_b200.GNN_cuda_common import npz_utils


def test_gcn_flag_defaults_match_reference():
    a = gcn_inference.build_parser().parse_args([])
    assert (a.dataset, a.dim, a.num_layers, a.memory_mode, a.spmm_mode, a.gcn_kernel_impl) == \
        ("cora", 128, 2, "uvm", "plain", "legacy_fused")
    assert (a.warmup, a.iters, a.device, a.tf32, a.ft_host_alloc, a.prefetch_to) == (1, 5, "cuda:0", True, 0.0, "none")
    assert a.prefetch_pieces == 0  # the reference's prefetch before the loop
    assert a.preprocess_meta == "none" and a.pretouch_passes == 0 and a.hmm_mode == "plain"
    a = gcn_inference.build_parser().parse_args(["--no-tf32", "--activation", "device", "--spmm_mode", "optimized"])
    assert a.tf32 is False and a.activation == "device" and a.spmm_mode == "optimized"


def test_sage_gin_flags():
    a = graphsage_inference.build_parser().parse_args(["--dim", "256", "--weight", "device"])
    assert a.dim == 256 and a.weight == "device" and not hasattr(a, "activation")
    g = gin_inference.build_parser().parse_args(["--learn_eps"])
    assert g.learn_eps and g.num_layers == 2


def _run_gcn(argv):
    return gcn_inference.run_gcn_inference(framework_label="pyg", select_device=npz_utils.select_device,
                                           load_graph_features=npz_utils.load_pyg_graph_features_from_npz,
                                           load_kind="pyg", argv=argv)


def test_gcn_argument_errors(tmp_path):
    with pytest.raises(ValueError, match="only supports float32"):
        _run_gcn(["--amp", "--device", "cpu"])
    with pytest.raises(ValueError, match="weight expects one of"):
        _run_gcn(["--weight", "hmm", "--device", "cpu"])
    with pytest.raises(ValueError, match="activation expects one of"):
        _run_gcn(["--activation", "hmm", "--device", "cpu"])
    with pytest.raises(ValueError, match=r"\[0, 100\)"):
        _run_gcn(["--ft_host_alloc", "100", "--device", "cpu"])
    with pytest.raises(ValueError, match="requires a CUDA device"):
        _run_gcn(["--ft_host_alloc", "20", "--device", "cpu"])
    with pytest.raises(ValueError, match="'hmm' requires a CUDA device"):
        _run_gcn(["--ft_matrix", "hmm", "--weight", "device", "--device", "cpu"])
    with pytest.raises(ValueError, match="only accepts a dataset name"):
        _run_gcn(["--dataset", "a/b", "--memory_mode", "device", "--device", "cpu"])


def test_npz_roundtrip(tmp_path):
    src = torch.tensor([0, 1, 2, 2])
    dst = torch.tensor([1, 2, 0, 3])
    npz_utils.save_graph_npz(str(tmp_path / "t.npz"), src, dst, 5)
    ei, feats, n = npz_utils.load_pyg_graph_features_from_npz(str(tmp_path / "t.npz"), 16, False)
    assert n == 5 and feats.shape == (5, 16) and torch.equal(ei[0], src) and torch.equal(ei[1], dst)
    s, d, f2, n2 = npz_utils.load_dgl_graph_features_from_npz(str(tmp_path / "t.npz"), 8, True)
    assert n2 == 5 and f2.shape == (5, 8)
    with pytest.raises(FileNotFoundError):
        npz_utils.load_pyg_graph_features_from_npz(str(tmp_path / "missing.npz"), 8, False)


def test_phase_summary_cpu_timer():
    from gnn_cuda_b200.GNN_cuda_common.phase_summary import PhaseSummary
    ps = PhaseSummary(torch.device("cpu"))
    with ps.measure("spmm"):
        pass
    ps.record_iteration(("spmm",))
    assert ps.total_ns("spmm") >= 0.0
    ps.reset()
    assert ps.iteration_values("spmm") == []


def test_layer_plan_flags_and_order_rule():
    """--fuse_layers is off unless asked for; --layer_order auto transforms first
    exactly when a layer narrows (out_dim < in_dim)."""
    from gnn_cuda_b200.GNN_cuda_common import _driver as D
    for mod in (gcn_inference, graphsage_inference, gin_inference):
        a = mod.build_parser().parse_args([])
        assert a.fuse_layers is False and a.layer_order == "auto"
        a = mod.build_parser().parse_args(["--fuse_layers", "--layer_order", "aggregate_first"])
        assert a.fuse_layers is True and a.layer_order == "aggregate_first"
    assert D.transform_first("auto", 256, 128) and not D.transform_first("auto", 128, 128)
    assert not D.transform_first("auto", 128, 256)
    assert D.transform_first("transform_first", 128, 256) and not D.transform_first("aggregate_first", 256, 64)
    with pytest.raises(ValueError):
        D.transform_first("sideways", 1, 1)
    # on a host without CUDA every layer runs aggregate-first (or transform-first when it narrows)
    a = gcn_inference.build_parser().parse_args(["--fuse_layers"])
    cpu = torch.device("cpu")
    assert gcn_inference._layer_plan(a, 0, 128, 128, device=cpu, impl="legacy_fused",
                                     optimized_first=False) == "aggregate_first"
    assert gcn_inference._layer_plan(a, 0, 256, 128, device=cpu, impl="legacy_fused",
                                     optimized_first=False) == "transform_first"
    g = gin_inference.build_parser().parse_args(["--fuse_layers"])
    assert gin_inference._layer_plan(g, 128, 128, device=cpu) == "aggregate_first"
    s = graphsage_inference.build_parser().parse_args(["--layer_order", "transform_first"])
    assert graphsage_inference._layer_plan(s, 128, 128, device=cpu) == "transform_first"
