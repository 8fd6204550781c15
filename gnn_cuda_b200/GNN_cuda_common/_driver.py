"""Pieces shared by the three inference drivers (gcn / graphsage / gin).

The reference repeats these in each driver (e.g. gcn_inference.py:45-111 and
:195-284); here they live once. Flag names, defaults, help-hidden aliases and
memory-mode resolution order are the reference's; ``--seed`` is an addition
(seeds PyTorch's generator before weights and features are drawn).
"""
from __future__ import annotations

import argparse
import contextlib
import os
from dataclasses import dataclass

import torch
from torch import nn

from .allocator import COMPUTE_MEMORY_MODES, GRAPH_MEMORY_MODES, normalize_memory_mode, pointer_info

# the reference drivers' --data_root default (gcn_inference.py:197), kept so scripts that rely on it still work
DEFAULT_DATA_ROOT = "/root/workspace/mnt/dataset_npz"


def autocast_context(use_amp: bool, device: torch.device):
    if use_amp and device.type == "cuda":
        return torch.amp.autocast(device_type="cuda", dtype=torch.float16)
    return contextlib.nullcontext()


def cuda_profiler(device: torch.device, start: bool) -> None:
    if device.type != "cuda":
        return
    try:
        torch.cuda.synchronize(device)
        (torch.cuda.cudart().cudaProfilerStart if start else torch.cuda.cudart().cudaProfilerStop)()
    except Exception:
        pass


@contextlib.contextmanager
def nvtx_range(enabled: bool, name: str):
    if enabled and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        if enabled and torch.cuda.is_available():
            torch.cuda.nvtx.range_pop()


def configure_tf32(enabled: bool, device: torch.device) -> None:
    """The reference's --tf32 switch; it also selects TF32 tensor cores for gemm_forward_."""
    if device.type != "cuda":
        return
    torch.backends.cuda.matmul.allow_tf32 = bool(enabled)
    torch.backends.cudnn.allow_tf32 = bool(enabled)
    torch.set_float32_matmul_precision("high" if enabled else "highest")


def describe_memory(name: str, tensor: torch.Tensor) -> str:
    info = pointer_info(tensor)
    return (f"{name}:\tdevice={info.get('device_type')}:{info.get('device_index')} "
            f"type={info.get('pointer_type')} managed={info.get('is_managed')}")


def init_linear_params(in_dim: int, out_dim: int, *, bias: bool = True):
    """nn.Linear's default init; weight stored [in, out] (= Linear.weight^T)."""
    lin = nn.Linear(in_dim, out_dim, bias=bias)
    w = lin.weight.detach().t().contiguous().cpu()
    b = lin.bias.detach().contiguous().cpu() if bias else None
    return w, b


def layer_dims(in_dim: int, hidden_dim: int, out_dim: int, num_layers: int) -> list[tuple[int, int]]:
    n = max(1, int(num_layers))
    if n == 1:
        return [(in_dim, out_dim)]
    return [(in_dim, hidden_dim)] + [(hidden_dim, hidden_dim)] * (n - 2) + [(hidden_dim, out_dim)]


def base_parser(model: str) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser()
    p.add_argument("--dataset", type=str, default="cora", help="dataset name")
    p.add_argument("--data_root", type=str, default=os.environ.get("GNN_DATASET_ROOT", DEFAULT_DATA_ROOT),
                   help="directory containing <dataset>.npz")
    p.add_argument("--dim", type=int, default=128, help="base dim for input/hidden/output")
    p.add_argument("--feat_dim", type=int, default=None, help=argparse.SUPPRESS)
    p.add_argument("--hidden_dim", type=int, default=None, help=argparse.SUPPRESS)
    p.add_argument("--out_dim", type=int, default=None, help=argparse.SUPPRESS)
    p.add_argument("--num_layers", type=int, default=2, help=f"number of {model} layers")
    return p


def add_placement_flags(p: argparse.ArgumentParser, *, activation: bool) -> None:
    p.add_argument("--use_npz_features", action="store_true", help="use sparse features saved in npz if present")
    p.add_argument("--memory_mode", type=str, default="uvm",
                   help="shared fallback backend for adjacency/features/weight allocation: device, uvm, or hmm; "
                        "legacy aliases managed/torch_cuda are also accepted")
    p.add_argument("--graph_memory_mode", type=str, default=None, help=argparse.SUPPRESS)
    p.add_argument("--adj_matrix", type=str, default=None, help="adjacency backend for CSR inputs: device, uvm, hmm")
    p.add_argument("--ft_matrix", type=str, default=None, help="feature backend for node feature tensors: device, uvm, hmm")
    p.add_argument("--weight", type=str, default=None, help="compute backend for weights/outputs/scratch: device or uvm")
    if activation:
        p.add_argument("--activation", type=str, default=None,
                       help="activation backend for aggregation/output buffers: device or uvm")
    p.add_argument("--compute_memory_mode", type=str, default=None, help=argparse.SUPPRESS)


def add_runtime_flags(p: argparse.ArgumentParser) -> None:
    p.add_argument("--preferred_location", type=str, default="none", choices=["none", "cpu", "cuda"],
                   help="UVM preferred location hint")
    p.add_argument("--accessed_by_cpu", action="store_true", help="mark UVM tensors as CPU-accessible")
    p.add_argument("--accessed_by_cuda", action="store_true", help="mark UVM tensors as GPU-accessible")
    p.add_argument("--read_mostly_graph", action="store_true", help="mark graph structures as read-mostly")
    p.add_argument("--prefetch_to", type=str, default="none", choices=["none", "cpu", "cuda"],
                   help="prefetch UVM tensors before compute")
    p.add_argument("--amp", action="store_true", help="reserved; CUDA prototype currently runs fp32")
    p.add_argument("--tf32", action=argparse.BooleanOptionalAction, default=True,
                   help="allow TF32 Tensor Core path for float32 GEMM on CUDA")
    p.add_argument("--nvtx", action="store_true", help="enable NVTX ranges for profiling")
    p.add_argument("--warmup", type=int, default=1, help="warmup iterations")
    p.add_argument("--iters", type=int, default=5, help="inference iterations")
    p.add_argument("--device", type=str, default="cuda:0", help="device string")
    p.add_argument("--seed", type=int, default=None, help="seed PyTorch's generator (weights, random features)")
    p.add_argument("--fuse_layers", action=argparse.BooleanOptionalAction, default=False,
                   help="aggregate and transform each layer in one kernel when the widths allow it: the same "
                        "results as the separate calls with no [N, F] aggregate (or GIN hidden) buffer, for graphs "
                        "whose buffers would not fit; slower than the separate calls on one B200 (8.8 vs 3.6 ms per "
                        "GCN layer of the 2.45M-node products-shaped graph)")
    p.add_argument("--layer_order", type=str, default="auto", choices=["auto", "aggregate_first", "transform_first"],
                   help="per layer: aggregate then transform (the reference's order), transform then aggregate, or "
                        "auto: transform first exactly when the layer narrows (out_dim < in_dim), which gathers "
                        "out_dim-wide rows instead of in_dim-wide ones (results within the TF32 tolerance)")


def transform_first(order: str, in_dim: int, out_dim: int) -> bool:
    """Whether a layer multiplies by W before aggregating. Aggregation is linear,
    so A·(X·W) = (A·X)·W; transforming first gathers out_dim-wide rows, which
    pays exactly when the layer narrows."""
    if order == "transform_first":
        return True
    if order == "aggregate_first":
        return False
    if order != "auto":
        raise ValueError("layer_order must be auto, aggregate_first or transform_first")
    return int(out_dim) < int(in_dim)


@dataclass
class Placement:
    shared: str
    adj: str
    ft: str
    weight: str
    activation: str


def resolve_placement(args, *, with_activation: bool) -> Placement:
    """--adj_matrix/--ft_matrix -> --graph_memory_mode -> --memory_mode; --weight/--activation."""
    shared = normalize_memory_mode(args.memory_mode, allow_hmm=True)
    graph_fallback = args.graph_memory_mode or shared
    adj = normalize_memory_mode(args.adj_matrix or graph_fallback, allow_hmm=True)
    ft = normalize_memory_mode(args.ft_matrix or graph_fallback, allow_hmm=True)
    try:
        weight = normalize_memory_mode(args.weight or args.compute_memory_mode or shared, allow_hmm=False)
    except ValueError as exc:
        raise ValueError(
            f"weight expects one of {COMPUTE_MEMORY_MODES}; use --adj_matrix/--ft_matrix hmm with --weight uvm/device"
        ) from exc
    activation = weight
    if with_activation:
        try:
            activation = normalize_memory_mode(args.activation or weight, allow_hmm=False)
        except ValueError as exc:
            raise ValueError(
                f"activation expects one of {COMPUTE_MEMORY_MODES}; HMM outputs are not supported by the current "
                "dense path") from exc
    args.memory_mode, args.adj_matrix, args.ft_matrix, args.weight = shared, adj, ft, weight
    if with_activation:
        args.activation = activation
    return Placement(shared, adj, ft, weight, activation)


def check_hmm_device(placement: Placement, device: torch.device) -> None:
    if "hmm" in (placement.adj, placement.ft) and device.type != "cuda":
        raise ValueError(f"adj_matrix/ft_matrix expect one of {GRAPH_MEMORY_MODES} on CUDA; "
                         "'hmm' requires a CUDA device")


def fill_dims(args) -> None:
    base = int(args.dim)
    args.feat_dim = base if args.feat_dim is None else args.feat_dim
    args.hidden_dim = base if args.hidden_dim is None else args.hidden_dim
    args.out_dim = base if args.out_dim is None else args.out_dim
