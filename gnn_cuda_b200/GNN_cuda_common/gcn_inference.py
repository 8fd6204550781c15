"""GCN inference driver (reference: GNN_cuda_common/gcn_inference.py:188-686).

Same flags, memory placement, UVM hints/prefetch, ``--ft_host_alloc`` device
reserve and printed report as the reference. Per layer:
    agg = Â·x                    (spmm_gcn_forward_ / spmm_pyg_gcn_forward_)
    out = relu?(agg·W + b)       (linear_forward_: tcgen05 GEMM, bias+ReLU fused)
ReLU on every layer but the last. The reference ran GEMM and bias/ReLU as two
launches and synchronised after every phase; here the phases only record
CUDA events, so one forward is a single stream of launches.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import torch

from .. import _native as N
from .. import partition
from . import _driver as D
from . import native_ops
from .agg_ops import bias_relu_forward_, gemm_forward_, linear_forward_
from .fused_ops import fused_supported, gcn_layer_forward_
from .allocator import (
    ManagedAllocationConfig,
    allocate_empty,
    allocate_like_mode,
    apply_managed_policy,
    is_uvm_mode,
    prefetch_managed,
    prefetch_rows_in_order,
    uses_cuda_memory_hints,
)
from .gcn_ops import spmm_gcn_forward_, stage_feature_rows_
from .graph_utils import (
    apply_node_permutation,
    build_gcn_normalized_csr,
    build_pyg_gcn_weighted_csr,
    default_gcn_preprocess_meta_path,
    resolve_dataset_path,
)
from .phase_summary import PhaseSummary, print_summary_report
from .pyg_gcn_ops import spmm_pyg_gcn_forward_

PARTIAL_PREFETCH_FRACTION = 0.80
MIN_PARTIAL_PREFETCH_RUNTIME_SLACK_BYTES = 128 * 1024 * 1024


@dataclass
class LayerState:
    weight: torch.Tensor
    bias: torch.Tensor
    agg_buffer: torch.Tensor
    out_buffer: torch.Tensor


def _managed_hints(tensors, cfg: ManagedAllocationConfig, device, *, read_mostly: bool, prefetch: bool = True):
    for t in tensors:
        apply_managed_policy(t, device=device, preferred_location=cfg.preferred_location,
                             accessed_by_cpu=cfg.accessed_by_cpu, accessed_by_cuda=cfg.accessed_by_cuda,
                             read_mostly=read_mostly)
        if prefetch:
            prefetch_managed(t, location=cfg.prefetch_to, device=device)


def _layer_plan(args, idx: int, in_dim: int, out_dim: int, *, device, impl: str, optimized_first: bool) -> str:
    """How layer idx runs: "transform_first" (x·W, then aggregate; --layer_order),
    "fused" (one kernel for the aggregation and the transform; --fuse_layers,
    supported widths, TF32, the symmetric-normalisation kernels, not the first
    layer of spmm_mode=optimized) or "aggregate_first" (separate calls)."""
    if D.transform_first(str(args.layer_order), in_dim, out_dim):
        return "transform_first"
    if (bool(args.fuse_layers) and device.type == "cuda" and impl != "pyg_baseline"
            and not (idx == 0 and optimized_first) and fused_supported(in_dim, out_dim)):
        return "fused"
    return "aggregate_first"


def _make_layer_state(in_dim, out_dim, *, num_nodes, device, weight_mode, activation_mode, cfg,
                      plan: str = "aggregate_first") -> LayerState:
    w_cpu, b_cpu = D.init_linear_params(in_dim, out_dim)
    w = allocate_like_mode(w_cpu, memory_mode=weight_mode, device=device)
    b = allocate_like_mode(b_cpu, memory_mode=weight_mode, device=device)
    # the aggregate buffer: [N, in] (aggregate first), [N, out] (x·W first), none when fused
    agg_rows = 0 if plan == "fused" else num_nodes
    agg_cols = out_dim if plan == "transform_first" else in_dim
    agg = allocate_empty((agg_rows, agg_cols), dtype=torch.float32, device=device, memory_mode=activation_mode)
    out = allocate_empty((num_nodes, out_dim), dtype=torch.float32, device=device, memory_mode=activation_mode)
    if is_uvm_mode(weight_mode):
        _managed_hints((w, b), cfg, device, read_mostly=False)
    if is_uvm_mode(activation_mode):
        _managed_hints((agg, out), cfg, device, read_mostly=False)
    return LayerState(w, b, agg, out)


def _resolve_preprocess_meta_path(mode: str, *, dataset: str, data_root: str) -> str | None:
    if mode == "none":
        return None
    if mode == "auto":
        cand = default_gcn_preprocess_meta_path(dataset, data_root=data_root)
        return cand if Path(cand).exists() else None
    return mode


def build_parser():
    p = D.base_parser("GCN")
    D.add_placement_flags(p, activation=True)
    p.add_argument("--spmm_mode", type=str, default="plain", choices=["naive", "plain", "optimized"],
                   help="SpMM kernel variant: naive, plain, or optimized")
    p.add_argument("--gcn_kernel_impl", type=str, default="legacy_fused", choices=["legacy_fused", "pyg_baseline"],
                   help="GCN aggregation implementation: legacy fused normalization kernel or PyG-baseline-style "
                        "weighted CSR kernel")
    import argparse
    p.add_argument("--hmm_mode", type=str, default="plain", choices=["plain", "optimized"], help=argparse.SUPPRESS)
    p.add_argument("--preprocess_meta", type=str, default="none", help=argparse.SUPPRESS)
    p.add_argument("--pretouch_passes", type=int, default=0, help=argparse.SUPPRESS)
    D.add_runtime_flags(p)
    p.add_argument("--ft_host_alloc", type=float, default=0.0,
                   help="target percent of the feature matrix that should not fit in the remaining effective GPU memory")
    p.add_argument("--prefetch_pieces", type=int, default=0,
                   help="with --ft_matrix uvm and --prefetch_to cuda: instead of prefetching the features once before "
                        "the loop, prefetch them in this many row ranges on a side stream in every forward, and run "
                        "the first aggregation in as many row pieces, piece p starting when range p has arrived "
                        "(0: the reference's prefetch before the loop)")
    return p


def run_gcn_inference(*, framework_label: str, select_device: Callable[[str], torch.device], load_graph_features,
                      load_kind: str, argv: list[str] | None = None, capture: dict | None = None) -> int:
    args = build_parser().parse_args(argv)
    D.fill_dims(args)
    if args.seed is not None:
        torch.manual_seed(int(args.seed))
    device = select_device(args.device)
    D.configure_tf32(bool(args.tf32), device)
    if args.amp:
        raise ValueError("The CUDA GCN prototype only supports float32 today.")
    nvtx = bool(args.nvtx and device.type == "cuda")
    phases = PhaseSummary(device)
    place = D.resolve_placement(args, with_activation=True)
    print(args)
    D.check_hmm_device(place, device)

    spmm_mode = str(args.spmm_mode)
    impl = str(args.gcn_kernel_impl)
    if spmm_mode == "plain" and str(args.hmm_mode) == "optimized":
        spmm_mode = "optimized"
    spmm_kernel = "naive" if spmm_mode == "naive" else "plain_shared"
    cfg = ManagedAllocationConfig(preferred_location=str(args.preferred_location),
                                  accessed_by_cpu=bool(args.accessed_by_cpu),
                                  accessed_by_cuda=bool(args.accessed_by_cuda or device.type == "cuda"),
                                  read_mostly_graph=bool(args.read_mostly_graph), prefetch_to=str(args.prefetch_to))
    meta_path = _resolve_preprocess_meta_path(str(args.preprocess_meta), dataset=str(args.dataset),
                                              data_root=str(args.data_root))
    meta = None
    row_schedule = None
    edge_weight = None
    hot_pages = torch.empty((0,), dtype=torch.long)
    hot_cache_coverage = 0.0
    page_reuse_histogram = torch.empty((0,), dtype=torch.long)
    hot_cache = None
    hot_cutoff = 0
    hot_fraction = 0.0
    hot_access_coverage = 0.0
    rows_per_page = row_block_size = window_num_blocks = 1
    optimized_active = False
    reordered = False

    ft_host_alloc = float(args.ft_host_alloc)
    if ft_host_alloc < 0.0 or ft_host_alloc >= 100.0:
        raise ValueError("--ft_host_alloc expects a value in [0, 100)")
    reserve_on = ft_host_alloc > 0.0
    ft_initial = "cpu" if is_uvm_mode(place.ft) else "none"
    if reserve_on:
        if device.type != "cuda":
            raise ValueError("--ft_host_alloc requires a CUDA device")
        if place.ft == "device":
            raise ValueError("--ft_host_alloc is only meaningful with --ft_matrix uvm|hmm")

    # reserve bookkeeping (gcn_inference.py:316-350)
    rs = dict(device_bytes=0, target=0, feature_bytes=0, free_before=0, free_after=0, activated=0, activations=0,
              prefetch=0)
    reserve = {"tensor": None}

    def activate_reserve():
        if rs["device_bytes"] <= 0 or reserve["tensor"] is not None:
            return
        try:
            reserve["tensor"] = torch.empty((rs["device_bytes"],), dtype=torch.uint8, device=device)
        except RuntimeError as exc:
            gib = rs["device_bytes"] / float(1024 ** 3)
            raise RuntimeError(f"Failed to reserve {rs['device_bytes']} bytes ({gib:.3f} GiB) of extra device memory") \
                from exc
        rs["activated"] = int(reserve["tensor"].numel())
        rs["activations"] += 1
        torch.cuda.synchronize(device)
        rs["free_after"] = int(torch.cuda.mem_get_info(device)[0])

    def release_reserve():
        if reserve["tensor"] is None:
            return
        reserve["tensor"] = None
        if device.type == "cuda":
            torch.cuda.empty_cache()
            torch.cuda.synchronize(device)

    overlap_pieces = int(args.prefetch_pieces)
    if overlap_pieces < 0:
        raise ValueError("--prefetch_pieces expects a value >= 0")
    if overlap_pieces and not (device.type == "cuda" and uses_cuda_memory_hints(place.ft)
                               and cfg.prefetch_to == "cuda" and impl != "pyg_baseline"):
        overlap_pieces = 0  # only for unified-memory features prefetched to the GPU

    with phases.measure("graph_prep", use_cuda_events=False):
        graph_path = resolve_dataset_path(str(args.dataset), data_root=str(args.data_root))
        loaded = load_graph_features(graph_path, feat_dim=args.feat_dim, use_npz_features=args.use_npz_features)
        if load_kind == "pyg":
            edge_index, features_cpu, num_nodes = loaded
            src, dst = edge_index[0].contiguous(), edge_index[1].contiguous()
        elif load_kind == "dgl":
            src, dst, features_cpu, num_nodes = loaded
        else:
            raise ValueError(f"Unsupported load_kind: {load_kind}")
        num_edges = int(src.numel())

        if meta_path is not None:
            meta = torch.load(meta_path, map_location="cpu")
            if "perm" in meta and "inv_perm" in meta:
                perm = torch.as_tensor(meta["perm"], dtype=torch.long).contiguous()
                inv_perm = torch.as_tensor(meta["inv_perm"], dtype=torch.long).contiguous()
                if int(perm.numel()) != int(num_nodes) or int(inv_perm.numel()) != int(num_nodes):
                    raise ValueError(f"preprocess metadata {meta_path} is incompatible with dataset {args.dataset}")
                src, dst, features_cpu = apply_node_permutation(src, dst, features_cpu, perm=perm, inv_perm=inv_perm)
                reordered = True
        if spmm_mode == "optimized":
            if meta_path is None:
                raise ValueError("--spmm_mode optimized requires --preprocess_meta auto|<path>")
            row_schedule_cpu = torch.as_tensor(meta["row_schedule"], dtype=torch.long).contiguous()
            if int(row_schedule_cpu.numel()) != int(num_nodes):
                raise ValueError(f"preprocess metadata {meta_path} is incompatible with dataset {args.dataset}")
            hot_pages = torch.as_tensor(meta.get("hot_pages", []), dtype=torch.long).contiguous()
            hot_cache_coverage = float(meta.get("hot_coverage", 0.0))
            hot_cutoff = max(0, int(meta.get("hot_node_cutoff", 0)))
            hot_fraction = float(meta.get("hot_node_fraction", 0.0))
            hot_access_coverage = float(meta.get("hot_node_access_coverage", 0.0))
            page_reuse_histogram = torch.as_tensor(meta.get("page_reuse_histogram", []), dtype=torch.long).contiguous()
            rows_per_page = max(1, int(meta.get("rows_per_page", 1)))
            row_block_size = max(1, int(meta.get("row_block_size", 1)))
            window_num_blocks = max(1, int(meta.get("window_num_blocks", 1)))
            if place.ft not in {"hmm", "uvm"}:
                raise ValueError("--spmm_mode optimized currently requires --ft_matrix uvm|hmm")
            row_schedule = row_schedule_cpu.to(device=device, dtype=torch.long)

        features_cpu = features_cpu.contiguous().to(dtype=torch.float32)
        rs["feature_bytes"] = int(features_cpu.numel() * features_cpu.element_size())
        if impl == "pyg_baseline":
            wcsr = build_pyg_gcn_weighted_csr(src, dst, num_nodes=num_nodes, add_self_loops=True)
            row_ptr = allocate_like_mode(wcsr.row_ptr, memory_mode=place.adj, device=device)
            col_ind = allocate_like_mode(wcsr.col_ind, memory_mode=place.adj, device=device)
            edge_weight = allocate_like_mode(wcsr.edge_weight, memory_mode=place.adj, device=device)
            deg_inv_sqrt = None
            adj_tensors = (row_ptr, col_ind, edge_weight)
            spmm_kernel = f"{spmm_kernel}_pyg"
        else:
            csr = build_gcn_normalized_csr(src, dst, num_nodes=num_nodes, add_self_loops=True)
            row_ptr = allocate_like_mode(csr.row_ptr, memory_mode=place.adj, device=device)
            col_ind = allocate_like_mode(csr.col_ind, memory_mode=place.adj, device=device)
            deg_inv_sqrt = allocate_like_mode(csr.deg_inv_sqrt, memory_mode=place.adj, device=device)
            adj_tensors = (row_ptr, col_ind, deg_inv_sqrt)
        if uses_cuda_memory_hints(place.adj):
            _managed_hints(adj_tensors, cfg, device, read_mostly=cfg.read_mostly_graph)
        if row_schedule is not None and hot_cutoff > 0:
            hot_cache = torch.empty((hot_cutoff, int(features_cpu.size(1))), dtype=torch.float32, device=device)
            optimized_active = True

        dims = D.layer_dims(int(features_cpu.size(1)), int(args.hidden_dim), int(args.out_dim), int(args.num_layers))
        plans = [_layer_plan(args, idx, i, o, device=device, impl=impl, optimized_first=optimized_active)
                 for idx, (i, o) in enumerate(dims)]
        print(f"Layer plan: {', '.join(plans)}")
        layers = [_make_layer_state(i, o, num_nodes=int(num_nodes), device=device, weight_mode=place.weight,
                                    activation_mode=place.activation, cfg=cfg, plan=plan)
                  for (i, o), plan in zip(dims, plans)]
        if reserve_on:
            # the aggregation's scratch must exist before the reserve takes the free memory
            native_ops.ensure_workspace(device, int(num_nodes), int(col_ind.numel()))
            torch.cuda.synchronize(device)
            fit = max(0.0, (100.0 - ft_host_alloc) / 100.0)
            rs["target"] = int(rs["feature_bytes"] * fit)
            if cfg.prefetch_to == "cuda":
                if rs["target"] >= MIN_PARTIAL_PREFETCH_RUNTIME_SLACK_BYTES:
                    rs["prefetch"] = max(0, min(int(rs["target"] * PARTIAL_PREFETCH_FRACTION), rs["feature_bytes"]))
                else:
                    rs["prefetch"] = 0
            free_bytes, _ = torch.cuda.mem_get_info(device)
            rs["free_before"] = int(free_bytes)
            rs["device_bytes"] = max(0, int(free_bytes) - rs["target"] - rs["prefetch"])
            activate_reserve()

        features = allocate_like_mode(features_cpu, memory_mode=place.ft, device=device, uvm_initial_location=ft_initial)
        ft_preferred = cfg.preferred_location
        if uses_cuda_memory_hints(place.ft):
            ft_preferred = "cpu" if reserve_on and cfg.prefetch_to == "cuda" else cfg.preferred_location
            apply_managed_policy(features, device=device, preferred_location=ft_preferred,
                                 accessed_by_cpu=cfg.accessed_by_cpu, accessed_by_cuda=cfg.accessed_by_cuda,
                                 read_mostly=False)
            if ft_initial != "none":
                prefetch_managed(features, location=ft_initial, device=device)
                if device.type == "cuda":
                    torch.cuda.synchronize(device)
            if cfg.prefetch_to == "cuda":
                if not reserve_on:
                    rs["prefetch"] = rs["feature_bytes"]
                if overlap_pieces == 0:
                    prefetch_managed(features, location=cfg.prefetch_to, device=device,
                                     nbytes=rs["prefetch"] if reserve_on else None)
            else:
                prefetch_managed(features, location=cfg.prefetch_to, device=device)
        if hot_cache is not None:
            stage_feature_rows_(features, hot_cache)
        if optimized_active:
            spmm_kernel = f"optimized_pyg_{place.ft}" if impl == "pyg_baseline" else f"optimized_{place.ft}"

    # overlapped prefetch: row ranges of the features (the part that is prefetched)
    # and equal-entry row pieces of the first aggregation
    pieces, feat_ranges, piece_thr, pf_stream = [], [], 0, None
    if overlap_pieces and not (optimized_active or plans[0] != "aggregate_first"):
        row_bytes = int(features.size(1)) * features.element_size()
        prefix_rows = min(int(num_nodes), int(rs["prefetch"]) // max(1, row_bytes))
        step = -(-prefix_rows // overlap_pieces) if prefix_rows else 0
        feat_ranges = [(min(i * step, prefix_rows), min((i + 1) * step, prefix_rows)) for i in range(overlap_pieces)]
        bounds = partition.piece_bounds(row_ptr.to(torch.int64).cpu().numpy(), overlap_pieces)
        pieces = [partition.make_shard(row_ptr, col_ind, b0, b1) for b0, b1 in zip(bounds[:-1], bounds[1:])]
        piece_thr = int(N.lib().gnn_spmm_long_row_threshold(int(num_nodes), int(col_ind.numel())))
        pf_stream = torch.cuda.Stream(device)
        print(f"Overlapped prefetch: {len(feat_ranges)} feature ranges of {step} rows, {len(pieces)} row pieces")

    def aggregate_in_pieces(layer: LayerState, tag: str, x: torch.Tensor) -> None:
        """The first aggregation in row pieces, each waiting only for its feature range."""
        cur = torch.cuda.current_stream(device)
        pf_stream.wait_stream(cur)
        events = prefetch_rows_in_order(x, device=device, row_bounds=[r for r in feat_ranges if r[1] > r[0]],
                                        stream=pf_stream)
        old_thr = N.config_get("spmm.long_row_threshold")
        N.config_set("spmm.long_row_threshold", piece_thr)  # cut long rows as one whole-graph call does
        try:
            with D.nvtx_range(nvtx, f"{tag}/aggregation"):
                with phases.measure("spmm"):
                    for p_i, shard in enumerate(pieces):
                        if events:
                            cur.wait_event(events[min(p_i, len(events) - 1)])
                        partition.spmm_gcn_shard(shard, deg_inv_sqrt, x,
                                                 layer.agg_buffer[shard.row_begin:shard.row_end])
            if events:
                cur.wait_event(events[-1])
        finally:
            N.config_set("spmm.long_row_threshold", old_thr)

    feature_addr_start = int(features.data_ptr())
    feature_addr_end = feature_addr_start + rs["feature_bytes"]

    def aggregate(layer: LayerState, idx: int, tag: str, mode: str, x: torch.Tensor,
                  dst: torch.Tensor | None = None) -> None:
        dst = layer.agg_buffer if dst is None else dst
        with D.nvtx_range(nvtx, f"{tag}/aggregation"):
            with phases.measure("spmm"):
                first = idx == 0
                if plans[idx] == "fused":
                    # aggregation and transform in one kernel: the layer's output directly
                    gcn_layer_forward_(row_ptr, col_ind, deg_inv_sqrt, x, layer.weight, layer.bias, layer.out_buffer,
                                       relu=idx != len(layers) - 1)
                elif impl == "pyg_baseline":
                    spmm_pyg_gcn_forward_(row_ptr, col_ind, edge_weight, x, dst, spmm_mode=mode,
                                          optimized_backend=place.ft if first else "hmm",
                                          row_schedule=row_schedule if first else None,
                                          hot_feature_cache=hot_cache if first else None,
                                          hot_node_cutoff=hot_cutoff if first else 0)
                else:
                    spmm_gcn_forward_(row_ptr, col_ind, deg_inv_sqrt, x, dst, spmm_mode=mode,
                                      row_schedule=row_schedule if first else None,
                                      hot_feature_cache=hot_cache if first else None,
                                      hot_node_cutoff=hot_cutoff if first else 0)

    def forward_once() -> torch.Tensor:
        x = features
        for idx, layer in enumerate(layers):
            tag = f"layer{idx + 1}"
            mode = spmm_mode
            if idx == 0 and optimized_active:
                mode = "optimized"
            elif idx != 0 and mode == "optimized":
                mode = "plain"
            relu = idx != len(layers) - 1
            src, dst = x, None
            if plans[idx] == "transform_first":
                # A·(x·W): the narrower x·W rows are gathered; bias and ReLU after the aggregation
                with D.nvtx_range(nvtx, f"{tag}/dense_update"):
                    with phases.measure("gemm"):
                        gemm_forward_(x, layer.weight, layer.agg_buffer)
                src, dst = layer.agg_buffer, layer.out_buffer
            if idx == 0:
                activate_reserve()
                try:
                    if pieces:
                        aggregate_in_pieces(layer, tag, src)
                    else:
                        aggregate(layer, idx, tag, mode, src, dst)
                finally:
                    release_reserve()
            else:
                aggregate(layer, idx, tag, mode, src, dst)
            if plans[idx] == "aggregate_first":
                with D.nvtx_range(nvtx, f"{tag}/dense_update"):
                    with phases.measure("gemm"):
                        linear_forward_(layer.agg_buffer, layer.weight, layer.bias, layer.out_buffer, relu=relu)
            elif plans[idx] == "transform_first":
                with phases.measure("gemm"):
                    bias_relu_forward_(layer.out_buffer, layer.bias, relu)
            x = layer.out_buffer
        return x

    import time
    with torch.no_grad():
        for _ in range(max(0, int(args.pretouch_passes))):
            forward_once()
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
    print(f"Impl:\t{framework_label}_gcn_cuda")
    print(f"Adjacency Memory Mode:\t{place.adj}")
    print(f"Feature Memory Mode:\t{place.ft}")
    print(f"Feature Initial Location:\t{ft_initial}")
    print(f"Feature Prefetch To:\t{cfg.prefetch_to}")
    print(f"Feature Preferred Location:\t{ft_preferred if uses_cuda_memory_hints(place.ft) else 'none'}")
    print(f"Weight Memory Mode:\t{place.weight}")
    print(f"Activation Memory Mode:\t{place.activation}")
    print(f"GCN Kernel Impl:\t{impl}")
    print(f"SpMM Mode:\t{spmm_mode}")
    print(f"Pre-touch Passes:\t{int(args.pretouch_passes)}")
    print(f"Feature Host Alloc Target (%):\t{ft_host_alloc:.3f}")
    print(f"Feature Reserve Enabled:\t{reserve_on}")
    print(f"Feature Bytes:\t{rs['feature_bytes']}")
    print(f"Feature CUDA Prefetch Bytes:\t{rs['prefetch']}")
    print(f"Feature Address Start:\t{feature_addr_start}")
    print(f"Feature Address End:\t{feature_addr_end}")
    print(f"Target GPU Feature Bytes:\t{rs['target']}")
    print(f"Reserve Free Memory Before (GB):\t{rs['free_before'] / 1_000_000_000.0:.3f}")
    print(f"Reserve Free Memory After (GB):\t{rs['free_after'] / 1_000_000_000.0:.3f}")
    print(f"Reserved Device Memory (GB):\t{rs['device_bytes'] / 1_000_000_000.0:.3f}")
    print(f"Activated Reserved Device Memory (GB):\t{rs['activated'] / 1_000_000_000.0:.3f}")
    print(f"Reserve Activations:\t{rs['activations']}")
    print(f"SpMM Kernel:\t{spmm_kernel}")
    print(f"Preprocess Meta:\t{meta_path or 'none'}")
    print(f"Node Reorder:\t{reordered}")
    print(f"Page Rows Per Host Page:\t{rows_per_page}")
    print(f"Row Block Size:\t{row_block_size}")
    print(f"Window Num Blocks:\t{window_num_blocks}")
    print(f"Hot Feature Cache Pages:\t{int(hot_pages.numel())}")
    print(f"Hot Feature Cache Coverage:\t{hot_cache_coverage:.6f}")
    print(f"Hot Node Cutoff:\t{hot_cutoff}")
    print(f"Hot Node Fraction:\t{hot_fraction:.6f}")
    print(f"Hot Node Access Coverage:\t{hot_access_coverage:.6f}")
    print(f"Optimized Managed Active:\t{optimized_active}")
    if int(page_reuse_histogram.numel()) > 0:
        nz = torch.nonzero(page_reuse_histogram, as_tuple=False).flatten()
        if int(nz.numel()) > 0:
            head = nz[:8].tolist()
            print("Page Reuse Histogram Head:\t"
                  + ", ".join(f"{int(b)}->{int(page_reuse_histogram[int(b)].item())}" for b in head))
    print(f"Nodes:\t{num_nodes}")
    print(f"Edges:\t{num_edges}")
    print(D.describe_memory("row_ptr", row_ptr))
    print(D.describe_memory("col_ind", col_ind))
    if edge_weight is not None:
        print(D.describe_memory("edge_weight", edge_weight))
    else:
        print(D.describe_memory("deg_inv_sqrt", deg_inv_sqrt))
    print(D.describe_memory("features", features))
    print(D.describe_memory("weights_l0", layers[0].weight))
    if reserve["tensor"] is not None:
        print(D.describe_memory("reserve_tensor", reserve["tensor"]) + f" bytes={reserve['tensor'].numel()}")
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
