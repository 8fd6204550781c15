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


@dataclass
class PaddedLayout:
    """Rank r's rows sit at [r*max_rows, r*max_rows + rows_r) of a [world*max_rows, F] matrix.

    With every shard padded to max_rows, the between-layer exchange is one
    all_gather_into_tensor straight into the next layer's input. Global row g
    owned by rank r maps to padded id r*max_rows + (g - bounds[r]); the map is
    increasing, so CSR column order (and therefore every sum) is unchanged.
    """
    bounds: list[int]
    max_rows: int

    @property
    def world(self) -> int:
        return len(self.bounds) - 1

    @property
    def padded_rows(self) -> int:
        return self.world * self.max_rows

    def padded_ids(self, g: torch.Tensor) -> torch.Tensor:
        b = torch.as_tensor(self.bounds, dtype=torch.int64, device=g.device)
        owner = torch.searchsorted(b[1:-1], g.to(torch.int64), right=True)
        return owner * self.max_rows + (g.to(torch.int64) - b[owner])

    def pad_rows(self, full: torch.Tensor) -> torch.Tensor:
        """[N, ...] -> [world*max_rows, ...] with zero padding rows."""
        out = torch.zeros((self.padded_rows,) + tuple(full.shape[1:]), dtype=full.dtype, device=full.device)
        for r in range(self.world):
            b0, b1 = self.bounds[r], self.bounds[r + 1]
            out[r * self.max_rows:r * self.max_rows + (b1 - b0)] = full[b0:b1]
        return out

    def unpad_rows(self, padded: torch.Tensor) -> torch.Tensor:
        return torch.cat([padded[r * self.max_rows:r * self.max_rows + (self.bounds[r + 1] - self.bounds[r])]
                          for r in range(self.world)])


def make_padded_layout(row_ptr: np.ndarray, world: int) -> PaddedLayout:
    bounds = nnz_balanced_bounds(row_ptr, world)
    return PaddedLayout(bounds, max(1, max(bounds[i + 1] - bounds[i] for i in range(world))))


def make_padded_shard(row_ptr: torch.Tensor, col_ind: torch.Tensor, layout: PaddedLayout, rank: int) -> RowShard:
    """Rank `rank`'s rows with column ids rewritten to padded ids; row_begin is
    the shard's first padded row (r*max_rows)."""
    b0, b1 = layout.bounds[rank], layout.bounds[rank + 1]
    s = make_shard(row_ptr, col_ind, b0, b1)
    cols = layout.padded_ids(s.col_ind).to(torch.int32)
    base = rank * layout.max_rows
    return RowShard(base, base + (b1 - b0), s.row_ptr, cols.contiguous())


def gcn_forward_allgather(shard: RowShard, dis_pad: torch.Tensor, x_pad: torch.Tensor, weights: list[torch.Tensor],
                          biases: list[torch.Tensor], layout: PaddedLayout, bufs: dict, group=None,
                          timers: dict | None = None) -> torch.Tensor:
    """Multi-layer GCN over a padded-layout shard; one all_gather per layer boundary.

    bufs: 'agg' [rows, F], 'out' [max_rows, F] (padding rows zero), 'x_next'
    [world*max_rows, F]. Returns this rank's [rows, F] output rows.
    """
    x = x_pad
    rows = shard.num_rows
    layers = len(weights)
    for li in range(layers):
        ev = _mark(timers, "spmm_begin")
        spmm_gcn_shard(shard, dis_pad, x, bufs["agg"])
        _mark(timers, "spmm_end", ev)
        out = bufs["out"]
        native_ops.linear_forward_(bufs["agg"], weights[li], biases[li], out[:rows], li != layers - 1)
        if li == layers - 1:
            return out[:rows]
        dist.all_gather_into_tensor(bufs["x_next"], out, group=group)
        x = bufs["x_next"]
    return bufs["out"][:rows]


def _mark(timers: dict | None, key: str, begin=None):
    """Record a CUDA event for per-kernel timing (key 'spmm_begin' / 'spmm_end')."""
    if timers is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    if begin is not None:
        timers.setdefault("spmm", []).append((begin, ev))
    return ev
