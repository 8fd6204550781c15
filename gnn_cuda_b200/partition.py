"""Row-partitioned multi-GPU inference: one process per GPU, NCCL between layers.

SpMM rows are independent given the full input matrix, so rows shard with no
communication inside a layer. Each rank owns a contiguous row range chosen so
every rank holds about the same number of CSR entries (power-law graphs make
equal-row splits badly unbalanced), keeps the full feature matrix, and after
every layer except the last the ranks exchange their output rows so everyone
again holds the full [N, F] input of the next layer. Ranges are unequal, so the
exchange is one broadcast per owner rank into its slice of the full matrix
(every slice is a contiguous row block, so no repacking is needed).
Nothing here is model-specific; the GCN forward below is the benchmarked path.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from .GNN_cuda_common import native_ops


def nnz_balanced_bounds(row_ptr: np.ndarray, world: int) -> list[int]:
    """Row boundaries b[0]=0 < ... < b[world]=n with about nnz/world entries per range."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    n = row_ptr.shape[0] - 1
    nnz = int(row_ptr[-1])
    targets = [(nnz * r) // world for r in range(1, world)]
    inner = [int(np.searchsorted(row_ptr, t, side="left")) for t in targets]
    bounds = [0] + [min(max(b, 0), n) for b in inner] + [n]
    for i in range(1, len(bounds)):  # monotone even when one row holds more than a share
        bounds[i] = max(bounds[i], bounds[i - 1])
    return bounds


@dataclass
class RowShard:
    """Rows [row_begin, row_end) of a dst-major CSR, with global column ids."""
    row_begin: int
    row_end: int
    row_ptr: torch.Tensor  # [rows + 1], rebased to start at 0
    col_ind: torch.Tensor  # [shard nnz] int32, global column ids

    @property
    def num_rows(self) -> int:
        return self.row_end - self.row_begin

    @property
    def num_edges(self) -> int:
        return int(self.col_ind.numel())


def make_shard(row_ptr: torch.Tensor, col_ind: torch.Tensor, row_begin: int, row_end: int) -> RowShard:
    e0 = int(row_ptr[row_begin].item())
    e1 = int(row_ptr[row_end].item())
    rp = (row_ptr[row_begin:row_end + 1] - e0).contiguous()
    return RowShard(row_begin, row_end, rp, col_ind[e0:e1].contiguous())


def spmm_gcn_shard(shard: RowShard, deg_inv_sqrt: torch.Tensor, x_full: torch.Tensor, out: torch.Tensor) -> None:
    """out[rows of shard] = GCN aggregation over the full feature matrix."""
    assert out.shape == (shard.num_rows, x_full.shape[1]) and out.is_contiguous() and x_full.is_contiguous()
    dev = out.device
    idx = N.GNN_INDEX_INT64 if shard.row_ptr.dtype == torch.int64 else N.GNN_INDEX_INT32
    ws, wsb = native_ops._workspace(dev, N.lib().gnn_spmm_workspace_bytes(shard.num_rows, shard.num_edges))
    N.call("gnn_spmm_gcn_partition_forward", shard.row_ptr.data_ptr(), idx, shard.col_ind.data_ptr(),
           deg_inv_sqrt.data_ptr(), shard.row_begin, x_full.data_ptr(), out.data_ptr(), shard.num_rows,
           x_full.shape[0], shard.num_edges, x_full.shape[1], ws, wsb, native_ops._stream(dev))


def exchange_rows(local: torch.Tensor, full: torch.Tensor, bounds: list[int], rank: int, group=None) -> None:
    """full[b[r]:b[r+1]] <- rank r's `local`, for every rank r (NCCL or gloo)."""
    world = len(bounds) - 1
    for r in range(world):
        dst = full[bounds[r]:bounds[r + 1]]
        if r == rank:
            dst.copy_(local)
        if dst.numel():
            dist.broadcast(dst, src=r, group=group)


def gcn_forward_partitioned(shard: RowShard, deg_inv_sqrt: torch.Tensor, x_full: torch.Tensor,
                            weights: list[torch.Tensor], biases: list[torch.Tensor], bounds: list[int], rank: int,
                            bufs: dict, group=None, timers: dict | None = None) -> torch.Tensor:
    """Multi-layer GCN over a row shard: relu(Â X W + b) per layer, ReLU on all but the last.

    bufs holds preallocated 'agg' [rows, F], 'out0'/'out1' [rows, F] and 'x_next' [N, F].
    Returns this rank's rows of the final layer.
    """
    x = x_full
    layers = len(weights)
    for li in range(layers):
        agg = bufs["agg"]
        out = bufs["out0" if li % 2 == 0 else "out1"]
        ev = _mark(timers, "spmm_begin")
        spmm_gcn_shard(shard, deg_inv_sqrt, x, agg)
        _mark(timers, "spmm_end", ev)
        native_ops.linear_forward_(agg, weights[li], biases[li], out, li != layers - 1)
        if li != layers - 1:
            if len(bounds) > 2:
                exchange_rows(out, bufs["x_next"], bounds, rank, group)
                x = bufs["x_next"]
            else:
                x = out
        else:
            return out
    return out


def _mark(timers: dict | None, key: str, begin=None):
    """Record a CUDA event for per-kernel timing (key 'spmm_begin' / 'spmm_end')."""
    if timers is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    if begin is not None:
        timers.setdefault("spmm", []).append((begin, ev))
    return ev
