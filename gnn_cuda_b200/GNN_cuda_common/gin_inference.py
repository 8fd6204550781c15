"""GIN inference driver (reference: GNN_cuda_common/gin_inference.py:181-400).

Per layer (GINConv with an MLP Linear-ReLU-Linear):
    agg    = sum_{j in N(i)} x_j                 (spmm_sum_forward_)
    agg   += (1 + eps) * x                       (tensor_add_inplace_)
    hidden = relu(agg·W1 + b1)                   (linear_forward_, tcgen05 GEMM)
    out    = hidden·W2 + b2, ReLU when post_layer_relu and not the last layer
Same flags, placement and report as the reference. eps is read once per layer
at setup instead of with a device->host sync in every forward (the reference's
``layer.eps.item()``, gin_inference.py:332); the value is identical.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable

import torch

from . import _driver as D
from .agg_ops import bias_relu_forward_, gemm_forward_, linear_forward_, spmm_sum_forward_, tensor_add_inplace_
from .fused_ops import fused_supported, gin_layer_forward_
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
class GINLayerState:
    weight1: torch.Tensor
    bias1: torch.Tensor
    weight2: torch.Tensor
    bias2: torch.Tensor
    eps: torch.Tensor
    agg_buffer: torch.Tensor
    hidden_buffer: torch.Tensor
    out_buffer: torch.Tensor
    alpha: float = 1.0


def _apply_policy_if_needed(t, *, memory_mode, cfg, device, read_mostly, prefetch=True):
    if not uses_cuda_memory_hints(memory_mode):
        return
    apply_managed_policy(t, device=device, preferred_location=cfg.preferred_location,
                         accessed_by_cpu=cfg.accessed_by_cpu, accessed_by_cuda=cfg.accessed_by_cuda,
                         read_mostly=read_mostly)
    if prefetch:
        prefetch_managed(t, location=cfg.prefetch_to, device=device)


def _make_layer_state(in_dim, out_dim, *, num_nodes, device, memory_mode, cfg, learn_eps,
                      plan: str = "aggregate_first") -> GINLayerState:
    w1_cpu, b1_cpu = D.init_linear_params(in_dim, out_dim)
    w2_cpu, b2_cpu = D.init_linear_params(out_dim, out_dim)
    eps_cpu = torch.zeros((1,), dtype=torch.float32)
    # fused: no aggregate / hidden buffers; x·W1 first: the aggregate buffer holds x·W1 ([N, out])
    rows = 0 if plan == "fused" else num_nodes
    agg_cols = out_dim if plan == "transform_first" else in_dim
    st = GINLayerState(
        weight1=allocate_like_mode(w1_cpu, memory_mode=memory_mode, device=device),
        bias1=allocate_like_mode(b1_cpu, memory_mode=memory_mode, device=device),
        weight2=allocate_like_mode(w2_cpu, memory_mode=memory_mode, device=device),
        bias2=allocate_like_mode(b2_cpu, memory_mode=memory_mode, device=device),
        eps=allocate_like_mode(eps_cpu, memory_mode=memory_mode, device=device),
        agg_buffer=allocate_empty((rows, agg_cols), dtype=torch.float32, device=device, memory_mode=memory_mode),
        hidden_buffer=allocate_empty((rows, out_dim), dtype=torch.float32, device=device, memory_mode=memory_mode),
        out_buffer=allocate_empty((num_nodes, out_dim), dtype=torch.float32, device=device, memory_mode=memory_mode))
    if not learn_eps:
        st.eps.requires_grad_(False)
    for t in (st.weight1, st.bias1, st.weight2, st.bias2, st.eps, st.agg_buffer, st.hidden_buffer, st.out_buffer):
        _apply_policy_if_needed(t, memory_mode=memory_mode, cfg=cfg, device=device, read_mostly=False)
    st.alpha = 1.0 + float(st.eps.item())
    return st


def _layer_plan(args, in_dim: int, out_dim: int, *, device) -> str:
    """"transform_first" (x·W1 before the sum; --layer_order), "fused" (one
    kernel per layer; --fuse_layers, supported widths, TF32) or "aggregate_first"."""
    if D.transform_first(str(args.layer_order), in_dim, out_dim):
        return "transform_first"
    if bool(args.fuse_layers) and device.type == "cuda" and fused_supported(in_dim, out_dim, out_dim):
        return "fused"
    return "aggregate_first"


def build_parser():
    p = D.base_parser("GIN")
    p.add_argument("--learn_eps", action="store_true", help="allocate epsilon as a learnable-style state tensor")
    D.add_placement_flags(p, activation=False)
    D.add_runtime_flags(p)
    return p


def run_gin_inference(*, framework_label: str, select_device: Callable[[str], torch.device], load_graph_features,
                      load_kind: str, post_layer_relu: bool, argv: list[str] | None = None,
                      capture: dict | None = None) -> int:
    args = build_parser().parse_args(argv)
    D.fill_dims(args)
    if args.seed is not None:
        torch.manual_seed(int(args.seed))
    device = select_device(args.device)
    D.configure_tf32(bool(args.tf32), device)
    if args.amp:
        raise ValueError("The CUDA GIN prototype only supports float32 today.")
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
                                    learn_eps=bool(args.learn_eps), plan=plan)
                  for (i, o), plan in zip(dims, plans)]

    def forward_once() -> torch.Tensor:
        x = features
        for idx, layer in enumerate(layers):
            tag = f"layer{idx + 1}"
            relu_out = post_layer_relu and idx != len(layers) - 1
            if plans[idx] == "fused":
                # sum, + (1+eps)·x, Linear-ReLU-Linear in one kernel (same results as the calls below)
                with D.nvtx_range(nvtx, f"{tag}/fused"):
                    with phases.measure("spmm"):
                        gin_layer_forward_(row_ptr, col_ind, x, layer.alpha - 1.0, layer.weight1, layer.bias1,
                                           layer.weight2, layer.bias2, layer.out_buffer, relu_out)
                x = layer.out_buffer
                continue
            if plans[idx] == "transform_first":
                # sum and (1+eps)·x are linear: ((1+eps)x + Σx)·W1 = (1+eps)(x·W1) + Σ(x·W1)
                with phases.measure("gemm"):
                    gemm_forward_(x, layer.weight1, layer.agg_buffer)
                with phases.measure("spmm"):
                    spmm_sum_forward_(row_ptr, col_ind, layer.agg_buffer, layer.hidden_buffer,
                                      hmm_optimized=use_hmm_spmm)
                with phases.measure("epilogue"):
                    tensor_add_inplace_(layer.hidden_buffer, layer.agg_buffer, alpha=layer.alpha)
                    bias_relu_forward_(layer.hidden_buffer, layer.bias1, True)
                with phases.measure("gemm"):
                    linear_forward_(layer.hidden_buffer, layer.weight2, layer.bias2, layer.out_buffer, relu_out)
                x = layer.out_buffer
                continue
            with D.nvtx_range(nvtx, f"{tag}/aggregation"):
                with phases.measure("spmm"):
                    spmm_sum_forward_(row_ptr, col_ind, x, layer.agg_buffer, hmm_optimized=use_hmm_spmm)
            with D.nvtx_range(nvtx, f"{tag}/epilogue"):
                with phases.measure("epilogue"):
                    tensor_add_inplace_(layer.agg_buffer, x, alpha=layer.alpha)
            with D.nvtx_range(nvtx, f"{tag}/dense_update"):
                with phases.measure("gemm"):
                    linear_forward_(layer.agg_buffer, layer.weight1, layer.bias1, layer.hidden_buffer, True)
                    linear_forward_(layer.hidden_buffer, layer.weight2, layer.bias2, layer.out_buffer,
                                    post_layer_relu and idx != len(layers) - 1)
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
    print(f"Impl:\t{framework_label}_gin_cuda")
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
    print(D.describe_memory("weights1_l0", layers[0].weight1))
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
