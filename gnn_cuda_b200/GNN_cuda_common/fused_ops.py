"""One GNN layer in one pass: aggregation and dense transform without an [N, F]
aggregate buffer in device memory (libgnnb200 ``gnn_fused_aggregate_linear``).

The reference composes every layer from separate calls with full-size
buffers between them (``gcn_inference.py:534-600``: ``spmm_gcn_forward_`` into
``agg_buffer``, ``gemm_forward_``, ``bias_relu_forward_``;
``gin_inference.py:317-359``: ``spmm_sum_forward_``, ``tensor_add_inplace_``
and two ``linear_forward_``). These functions compute the same layers with
the same results — bit for bit equal to that sequence on this library's TF32
tensor-core path — while the aggregate only ever exists as a 128-row tile in
shared memory. They need the TF32 precision (``torch.backends.cuda.matmul.
allow_tf32``, the reference drivers' ``--tf32`` default) and widths the kernel
supports (``fused_supported``); callers fall back to the separate calls
otherwise.
"""
from __future__ import annotations

import torch

from .. import _native as N
from .native_ops import _check, _check_bias, _index_type, _stream, _workspace, gemm_precision


def fused_supported(feat_dim: int, width1: int, width2: int = 0) -> bool:
    """True when a fused layer with these widths runs here: TF32 precision
    selected, an sm_100 device, feat_dim in {32, 64, 96, 128}, widths in
    {32, 64, 128} and an output at least feat_dim wide."""
    if gemm_precision() != N.GNN_PRECISION_TF32 or not torch.cuda.is_available():
        return False
    return bool(N.lib().gnn_fused_layer_supported(int(feat_dim), int(width1), int(width2)))


def _check_inputs(row_ptr, col_ind, x, out, extra: dict) -> None:
    _check(out.is_cuda and x.is_cuda and row_ptr.is_cuda and col_ind.is_cuda, "out must be CUDA")
    for name, t in [("row_ptr", row_ptr), ("col_ind", col_ind), ("x", x), ("out", out)] + list(extra.items()):
        if t is not None:
            _check(t.is_contiguous(), f"{name} must be contiguous")
    _check(row_ptr.dtype in (torch.int32, torch.int64), "row_ptr must be int32")
    _check(col_ind.dtype == torch.int32, "col_ind must be int32")
    for name, t in [("x", x), ("out", out)] + list(extra.items()):
        if t is not None:
            _check(t.dtype == torch.float32, f"{name} must be float32")
    _check(x.dim() == 2 and out.dim() == 2, "x and out must be rank-2")
    _check(row_ptr.dim() == 1 and col_ind.dim() == 1, "row_ptr and col_ind must be rank-1")
    _check(row_ptr.numel() == out.size(0) + 1, "row_ptr length must be num_nodes + 1")
    _check(x.data_ptr() != out.data_ptr(), "out must not alias x")


def _call(row_ptr, col_ind, dis, aggregation: int, x, self_scale: float, add_self: bool, w1, b1, relu1: bool, w2, b2,
          relu2: bool, out, row_begin: int = 0) -> None:
    n = out.size(0)
    nnz = col_ind.numel()
    width1 = w1.size(1)
    width2 = 0 if w2 is None else w2.size(1)
    _check(w1.dim() == 2 and w1.size(0) == x.size(1), "Inner GEMM dimensions must match")
    if w2 is not None:
        _check(w2.dim() == 2 and w2.size(0) == width1, "Inner GEMM dimensions must match")
    _check(out.size(1) == (width2 or width1), "Output shape must match x @ weight")
    _check(fused_supported(x.size(1), width1, width2),
           "fused layer: unsupported widths or precision (see fused_supported)")
    dev = out.device
    with torch.cuda.device(dev):
        ws, wsb = _workspace(dev, N.lib().gnn_spmm_schedule_workspace_bytes(n, nnz))
        N.call("gnn_fused_aggregate_linear", row_ptr.data_ptr(), _index_type(row_ptr), col_ind.data_ptr() if nnz else None,
               None if dis is None else dis.data_ptr(), int(aggregation), int(row_begin), x.data_ptr(), n, x.size(0),
               nnz, x.size(1), float(self_scale), int(bool(add_self)), w1.data_ptr(),
               None if b1 is None or b1.numel() == 0 else b1.data_ptr(), width1, int(bool(relu1)),
               None if w2 is None else w2.data_ptr(), None if b2 is None or b2.numel() == 0 else b2.data_ptr(),
               width2, int(bool(relu2)), out.data_ptr(), ws, wsb, _stream(dev))


def gcn_layer_forward_(row_ptr, col_ind, deg_inv_sqrt, x, weight, bias, out, relu: bool = False) -> None:
    """out = relu?(Â·x·weight + bias) — spmm_gcn_forward_ then linear_forward_ in one pass."""
    _check_inputs(row_ptr, col_ind, x, out, {"deg_inv_sqrt": deg_inv_sqrt, "weight": weight})
    _check(x.size(0) == out.size(0), "x and out must have the same number of rows")
    _check(deg_inv_sqrt.numel() == x.size(0), "deg_inv_sqrt length must equal num_nodes")
    _check_bias(bias, out)
    _call(row_ptr, col_ind, deg_inv_sqrt, N.GNN_AGG_GCN, x, 1.0, False, weight, bias, relu, None, None, False, out)


def gin_layer_forward_(row_ptr, col_ind, x, eps: float, weight1, bias1, weight2, bias2, out,
                       relu_out: bool = False) -> None:
    """out = relu_out?(relu((Σx + (1+eps)·x)·W1 + b1)·W2 + b2) — spmm_sum_forward_,
    tensor_add_inplace_(agg, x, 1+eps) and two linear_forward_ calls in one pass."""
    _check_inputs(row_ptr, col_ind, x, out, {"weight1": weight1, "weight2": weight2})
    _check(x.size(0) == out.size(0), "x and out must have the same number of rows")
    _check_bias(bias2, out)
    if bias1 is not None and bias1.numel():
        _check(bias1.numel() == weight1.size(1), "bias length must equal output feature dimension")
    scale = float(torch.tensor(1.0 + float(eps), dtype=torch.float32))
    _call(row_ptr, col_ind, None, N.GNN_AGG_SUM, x, scale, True, weight1, bias1, True, weight2, bias2, relu_out, out)


def mean_linear_forward_(row_ptr, col_ind, x, weight, bias, out, relu: bool = False, reciprocal: bool = False) -> None:
    """out = relu?(mean(x)·weight + bias) — spmm_mean_forward_ (or the reciprocal
    variant) then linear_forward_ in one pass."""
    _check_inputs(row_ptr, col_ind, x, out, {"weight": weight})
    _check(x.size(0) == out.size(0), "x and out must have the same number of rows")
    _check_bias(bias, out)
    agg = N.GNN_AGG_MEAN_RECIPROCAL if reciprocal else N.GNN_AGG_MEAN
    _call(row_ptr, col_ind, None, agg, x, 1.0, False, weight, bias, relu, None, None, False, out)


def gin_layer_row_chunks_(row_ptr, col_ind, x, eps: float, weight1, bias1, weight2, bias2, out,
                          relu_out: bool = False, chunks: int = 16) -> None:
    """The GIN layer of gin_layer_forward_ as the separate calls (spmm_sum_forward_,
    tensor_add_inplace_, two linear_forward_) applied to `chunks` row ranges in turn,
    so the aggregate and hidden matrices only ever hold one range's rows.

    Same bits as the separate calls on the whole graph (and so as the fused
    kernel): each range is aggregated with the whole graph's long-row threshold,
    and every other step is row-wise. It costs two [N / chunks, F] buffers; on
    one B200 it was slower than the fused kernel on the 111M-node papers-shaped
    graph (370 against 288 ms per layer, 32 ranges)."""
    from .native_ops import linear_forward_, tensor_add_inplace_
    _check_inputs(row_ptr, col_ind, x, out, {"weight1": weight1, "weight2": weight2})
    _check(x.size(0) == out.size(0), "x and out must have the same number of rows")
    _check(x.size(1) == weight1.size(0) and weight1.size(1) == weight2.size(0) and out.size(1) == weight2.size(1),
           "Inner GEMM dimensions must match")
    n, f, nnz = out.size(0), x.size(1), col_ind.numel()
    if n == 0:
        return
    lib = N.lib()
    dev = out.device
    rows = -(-n // max(1, int(chunks)))
    agg = torch.empty(rows, f, device=dev)
    hid = torch.empty(rows, weight1.size(1), device=dev)
    alpha = float(torch.tensor(1.0 + float(eps), dtype=torch.float32))
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", int(lib.gnn_spmm_long_row_threshold(n, nnz)))
    starts = list(range(0, n, rows))
    offs = row_ptr[torch.tensor(starts + [n], device=row_ptr.device)].to(torch.int64).cpu().tolist()
    try:
        with torch.cuda.device(dev):
            for i, r0 in enumerate(starts):
                m = min(n, r0 + rows) - r0
                m_nnz = offs[i + 1] - offs[i]
                ws, wsb = _workspace(dev, lib.gnn_spmm_schedule_workspace_bytes(m, m_nnz))
                # rows [r0, r0 + m): row_ptr from entry r0 on (its offsets index col_ind as they are)
                N.call("gnn_spmm_sum_forward", row_ptr.data_ptr() + r0 * row_ptr.element_size(),
                       _index_type(row_ptr), col_ind.data_ptr() if nnz else None, x.data_ptr(), agg.data_ptr(), m,
                       m_nnz, f, ws, wsb, _stream(dev))
                tensor_add_inplace_(agg[:m], x[r0:r0 + m], alpha)
                linear_forward_(agg[:m], weight1, bias1, hid[:m], True)
                linear_forward_(hid[:m], weight2, bias2, out[r0:r0 + m], relu_out)
    finally:
        N.config_set("spmm.long_row_threshold", old)
