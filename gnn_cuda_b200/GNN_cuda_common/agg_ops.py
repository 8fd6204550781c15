"""Aggregation / dense ops with the reference's Python signatures
(GNN_cuda_common/agg_ops.py:9-63), backed by libgnnb200.so."""
from __future__ import annotations

import torch

from .loader import load_agg_module


def spmm_sum_forward_(row_ptr: torch.Tensor, col_ind: torch.Tensor, x: torch.Tensor, out: torch.Tensor, *,
                      hmm_optimized: bool = False) -> None:
    mod = load_agg_module()
    (mod.spmm_sum_hmm_forward_ if hmm_optimized else mod.spmm_sum_forward_)(row_ptr, col_ind, x, out)


def spmm_mean_forward_(row_ptr: torch.Tensor, col_ind: torch.Tensor, x: torch.Tensor, out: torch.Tensor, *,
                       hmm_optimized: bool = False) -> None:
    """hmm_optimized selects the reciprocal-multiply mean of the reference's hmm kernel."""
    mod = load_agg_module()
    (mod.spmm_mean_hmm_forward_ if hmm_optimized else mod.spmm_mean_forward_)(row_ptr, col_ind, x, out)


def gemm_forward_(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor) -> None:
    load_agg_module().gemm_forward_(x, weight, out)


def bias_relu_forward_(out: torch.Tensor, bias: torch.Tensor, relu: bool = False) -> None:
    load_agg_module().bias_relu_forward_(out, bias, bool(relu))


def linear_forward_(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, out: torch.Tensor,
                    relu: bool = False) -> None:
    """One launch: GEMM with bias and ReLU fused into its epilogue (the reference ran two)."""
    load_agg_module().linear_forward_(x, weight, bias, out, bool(relu))


def tensor_add_inplace_(dst: torch.Tensor, src: torch.Tensor, alpha: float = 1.0) -> None:
    load_agg_module().tensor_add_inplace_(dst, src, float(alpha))


def relu_inplace_(tensor: torch.Tensor) -> None:
    load_agg_module().relu_inplace_(tensor)
