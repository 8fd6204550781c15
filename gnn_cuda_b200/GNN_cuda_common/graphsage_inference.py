"""GraphSAGE-mean inference driver (reference: GNN_cuda_common/graphsage_inference.py:177-395).

Per layer (SAGEConv with mean aggregation, lin_l(mean) + lin_r(x)):
    agg  = mean_{j in N(i)} x_j                  (spmm_mean_forward_)
    out  = agg·W_neigh + b_neigh                 (linear_forward_, tcgen05 GEMM)
    root = x·W_root                              (gemm_forward_)
    out += root ; ReLU on all but the last layer (tensor_add_inplace_, relu_inplace_)
Same flags, placement and report as the reference; the reference's separate
bias pass after each GEMM is fused into the GEMM epilogue.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable

import torch

from . import _driver as D
from .agg_ops import (
    bias_relu_forward_,
    gemm_forward_,
    linear_forward_,
    relu_inplace_,
    spmm_mean_forward_,
    tensor_add_inplace_,
)
from .fused_ops import fused_supported, mean_linear_forward_
from .allocator import (
    ManagedAllocationConfig,
    allocate_empty,
    allocate_like_mode,
    apply_managed_policy,
    is_uvm_mode,
    prefers_hmm_spmm,
    prefetch_managed,
    uses_cuda_memory_hints,
)
from .graph_utils import build_plain_csr, load_src_dst_features, resolve_dataset_path
from .phase_summary import PhaseSummary, print_summary_report


@dataclass
class GraphSAGELayerState:
    weight_neigh: torch.Tensor
    bias_neigh: torch.Tensor
    weight_root: torch.Tensor
    bias_root: torch.Tensor
    agg_buffer: torch.Tensor
    root_buffer: torch.Tensor
    out_buffer: torch.Tensor


def _apply_policy_if_needed(t, *, memory_mode, cfg, device, read_mostly, prefetch=True):
    if not uses_cuda_memory_hints(memory_mode):
        return
    apply_managed_policy(t, device=device, preferred_location=cfg.preferred_location,
                         accessed_by_cpu=cfg.accessed_by_cpu, accessed_by_cuda=cfg.accessed_by_cuda,
                         read_mostly=read_mostly)
    if prefetch:
        prefetch_managed(t, location=cfg.prefetch_to, device=device)


def _layer_plan(args, in_dim: int, out_dim: int, *, device) -> str:
    """The neighbour half mean(x)·W_n + b_n: "transform_first" (mean of x·W_n;
    --layer_order), "fused" (one kernel; --fuse_layers, supported widths, TF32)
    or "aggregate_first"."""
    if D.transform_first(str(args.layer_order), in_dim, out_dim):
        return "transform_first"
    if bool(args.fuse_layers) and device.type == "cuda" and fused_supported(in_dim, out_dim):
        return "fused"
    return "aggregate_first"


def _make_layer_state(in_dim, out_dim, *, num_nodes, device, memory_mode, cfg,
                      plan: str = "aggregate_first") -> GraphSAGELayerState:
    wn_cpu, bn_cpu = D.init_linear_params(in_dim, out_dim, bias=True)
    wr_cpu, _ = D.init_linear_params(in_dim, out_dim, bias=False)
    br_cpu = torch.zeros((out_dim,), dtype=torch.float32)
    st = GraphSAGELayerState(
        weight_neigh=allocate_like_mode(wn_cpu, memory_mode=memory_mode, device=device),
        bias_neigh=allocate_like_mode(bn_cpu, memory_mode=memory_mode, device=device),
        weight_root=allocate_like_mode(wr_cpu, memory_mode=memory_mode, device=device),
        bias_root=allocate_like_mode(br_cpu, memory_mode=memory_mode, device=device),
        agg_buffer=allocate_empty((0 if plan == "fused" else num_nodes, out_dim if plan == "transform_first" else in_dim),
                                  dtype=torch.float32, device=device, memory_mode=memory_mode),
        root_buffer=allocate_empty((num_nodes, out_dim), dtype=torch.float32, device=device, memory_mode=memory_mode),
        out_buffer=allocate_empty((num_nodes, out_dim), dtype=torch.float32, device=device, memory_mode=memory_mode))
    for t in (st.weight_neigh, st.bias_neigh, st.weight_root, st.bias_root, st.agg_buffer, st.root_buffer,
              st.out_buffer):
        _apply_policy_if_needed(t, memory_mode=memory_mode, cfg=cfg, device=device, read_mostly=False)
    return st


def build_parser():
    p = D.base_parser("GraphSAGE")
    D.add_placement_flags(p, activation=False)
    D.add_runtime_flags(p)
    return p


def run_graphsage_inference(*, framework_label: str, select_device: Callable[[str], torch.device],
                            load_graph_features, load_kind: str, argv: list[str] | None = None,
                            capture: dict | None = None) -> int:
    args = build_parser().parse_args(argv)
    D.fill_dims(args)
    if args.seed is not None:
        torch.manual_seed(int(args.seed))
    device = select_device(args.device)
    D.configure_tf32(bool(args.tf32), device)
    if args.amp:
        raise ValueError("The CUDA GraphSAGE prototype only supports float32 today.")
    nvtx = bool(args.nvtx and device.type == "cuda")
    phases = PhaseSummary(device)
    place = D.resolve_placement(args, with_activation=False)
    print(args)
    ft_initial = "cpu" if is_uvm_mode(place.ft) else "none"
    D.check_hmm_device(place, device)
    use_hmm_spmm = prefers_hmm_spmm(place.adj, place.ft)
    spmm_kernel = "hmm_optimized" if use_hmm_spmm else "baseline"
    cfg = ManagedAllocationConfig(preferred_location=str(args.preferred_location),
                                  accessed_by_cpu=bool(args.accessed_by_cpu),
                                  accessed_by_cuda=bool(args.accessed_by_cuda or device.type == "cuda"),
                                  read_mostly_graph=bool(args.read_mostly_graph), prefetch_to=str(args.prefetch_to))

    with phases.measure("graph_prep", use_cuda_events=False):
        graph_path = resolve_dataset_path(str(args.dataset), data_root=str(args.data_root))
        loaded = load_graph_features(graph_path, feat_dim=args.feat_dim, use_npz_features=args.use_npz_features)
        src, dst, features_cpu, num_nodes = load_src_dst_features(loaded, load_kind=load_kind)
        num_edges = int(src.numel())
        csr = build_plain_csr(src, dst, num_nodes=num_nodes, add_self_loops=False, transpose_for_incoming=True)
        features_cpu = features_cpu.contiguous().to(dtype=torch.float32)
        row_ptr = allocate_like_mode(csr.row_ptr, memory_mode=place.adj, device=device)
        col_ind = allocate_like_mode(csr.col_ind, memory_mode=place.adj, device=device)
        features = allocate_like_mode(features_cpu, memory_mode=place.ft, device=device, uvm_initial_location=ft_initial)
        for t in (row_ptr, col_ind):
            _apply_policy_if_needed(t, memory_mode=place.adj, cfg=cfg, device=device, read_mostly=cfg.read_mostly_graph)
        _apply_policy_if_needed(features, memory_mode=place.ft, cfg=cfg, device=device, read_mostly=False,
                                prefetch=False)
        if uses_cuda_memory_hints(place.ft):
            if ft_initial != "none":
                prefetch_managed(features, location=ft_initial, device=device)
                if device.type == "cuda":
                    torch.cuda.synchronize(device)
            prefetch_managed(features, location=cfg.prefetch_to, device=device)
        dims = D.layer_dims(int(features.size(1)), int(args.hidden_dim), int(args.out_dim), int(args.num_layers))
        plans = [_layer_plan(args, i, o, device=device) for i, o in dims]
        print(f"Layer plan: {', '.join(plans)}")
        layers = [_make_layer_state(i, o, num_nodes=int(num_nodes), device=device, memory_mode=place.weight, cfg=cfg,
                                    plan=plan)
                  for (i, o), plan in zip(dims, plans)]

    def forward_once() -> torch.Tensor:
        x = features
        for idx, layer in enumerate(layers):
            tag = f"layer{idx + 1}"
            plan = plans[idx]
            if plan == "fused":
                # mean aggregation and agg·W_n + b_n in one kernel (same results as the two calls)
                with D.nvtx_range(nvtx, f"{tag}/fused"):
                    with phases.measure("spmm"):
                        mean_linear_forward_(row_ptr, col_ind, x, layer.weight_neigh, layer.bias_neigh,
                                             layer.out_buffer, False, use_hmm_spmm)
            elif plan == "transform_first":
                # mean is linear: mean(x)·W_n = mean(x·W_n), gathering out_dim-wide rows
                with phases.measure("gemm"):
                    gemm_forward_(x, layer.weight_neigh, layer.agg_buffer)
                with phases.measure("spmm"):
                    spmm_mean_forward_(row_ptr, col_ind, layer.agg_buffer, layer.out_buffer, hmm_optimized=use_hmm_spmm)
                with phases.measure("epilogue"):
                    bias_relu_forward_(layer.out_buffer, layer.bias_neigh, False)
            else:
                with D.nvtx_range(nvtx, f"{tag}/aggregation"):
                    with phases.measure("spmm"):
                        spmm_mean_forward_(row_ptr, col_ind, x, layer.agg_buffer, hmm_optimized=use_hmm_spmm)
            with D.nvtx_range(nvtx, f"{tag}/dense_update"):
                with phases.measure("gemm"):
                    if plan == "aggregate_first":
                        linear_forward_(layer.agg_buffer, layer.weight_neigh, layer.bias_neigh, layer.out_buffer,
                                        False)
                    gemm_forward_(x, layer.weight_root, layer.root_buffer)
                with phases.measure("epilogue"):
                    tensor_add_inplace_(layer.out_buffer, layer.root_buffer, alpha=1.0)
                    if idx != len(layers) - 1:
                        relu_inplace_(layer.out_buffer)
            x = layer.out_buffer
        return x

    with torch.no_grad():
        for _ in range(args.warmup):
            forward_once()
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        phases.reset()
        if capture is not None and capture.get("on_measure_begin"):
            capture["on_measure_begin"]()
        D.cuda_profiler(device, True)
        start = time.perf_counter()
        output = features
        for _ in range(args.iters):
            with D.nvtx_range(nvtx, "iteration"):
                output = forward_once()
            phases.record_iteration(("spmm", "gemm", "epilogue"))
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        elapsed = time.perf_counter() - start
        if capture is not None and capture.get("on_measure_end"):
            capture["on_measure_end"]()
        D.cuda_profiler(device, False)

    print(f"Graph:\t{graph_path}")
    print(f"Impl:\t{framework_label}_graphsage_cuda")
    print(f"Adjacency Memory Mode:\t{place.adj}")
    print(f"Feature Memory Mode:\t{place.ft}")
    print(f"Feature Initial Location:\t{ft_initial}")
    print(f"Feature Prefetch To:\t{cfg.prefetch_to}")
    print(f"Weight Memory Mode:\t{place.weight}")
    print(f"SpMM Kernel:\t{spmm_kernel}")
    print(f"Nodes:\t{num_nodes}")
    print(f"Edges:\t{num_edges}")
    print(D.describe_memory("row_ptr", row_ptr))
    print(D.describe_memory("col_ind", col_ind))
    print(D.describe_memory("features", features))
    print(D.describe_memory("weights_neigh_l0", layers[0].weight_neigh))
    print(D.describe_memory("output", output))
    if capture is not None:  # test hook: the final output and everything needed to recompute it
        capture.update(feature_range=(int(features.data_ptr()),
                                      int(features.data_ptr()) + features.numel() * features.element_size()),
                       spmm_avg_ns=phases.avg_ns("spmm", iters=int(args.iters)), iters=int(args.iters))
        capture.update(output=output.detach().cpu(), features=features.detach().cpu(), layers=layers,
                       row_ptr=row_ptr.detach().cpu(), col_ind=col_ind.detach().cpu(), num_nodes=num_nodes)
    print(f"Output Sum:\t{float(output.sum().item()):.6f}")
    infer_avg_ns = elapsed * 1e9 / args.iters
    print(f"Infer (ns):\t{infer_avg_ns:.3f}")
    print_summary_report(phases, iters=int(args.iters), infer_avg_ns=infer_avg_ns)
    return 0
