"""Row-partitioned multi-GPU inference: one process per GPU, NCCL between layers.

SpMM rows are independent given the full input matrix, so rows shard with no
communication inside a layer. Each rank owns a contiguous row range chosen so
every rank carries about the same aggregation cost — its CSR entries plus a
measured per-row cost (power-law graphs make equal-row splits badly
unbalanced) — keeps the full feature matrix, and after
every layer except the last the ranks exchange their output rows so everyone
again holds the full [N, F] input of the next layer.

Three exchanges are provided, all bit-identical to the one-GPU forward at a
fixed long-row threshold. `gcn_forward_push` (the benchmarked path) writes each
layer's output rows straight into the rank's rows of an IPC-mapped copy of the
next layer's input and sends every peer exactly the rows its CSR reads (the
halo): stored by the transform's own epilogue (`push_masks`), by a push kernel
after it, or by copy engines, with one small NCCL all_reduce per layer
boundary as the barrier; its steps can be captured and replayed as CUDA graphs
(`PushForwardGraphs`). `gcn_forward_allgather` renumbers rows into a padded
chunk-major layout and exchanges each piece with an asynchronous NCCL
all_gather. `gcn_forward_partitioned` keeps global row ids and broadcasts each
owner's row range.
"""
from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from .GNN_cuda_common import native_ops


# Aggregation cost of one row relative to one CSR entry, for balancing ranks:
# measured on B200 with the products-shaped GCN (F = 128) split into two
# equal-entry shards, time = a * entries + b * rows gives b / a ~ 6 (each row
# also writes a 512-byte output row and reads its bounds and scale).
ROW_COST_IN_ENTRIES = 6


def nnz_balanced_bounds(row_ptr: np.ndarray, world: int, row_cost: float = 0.0) -> list[int]:
    """Row boundaries b[0]=0 <= ... <= b[world]=n giving every range about the same
    cost, where a range costs its CSR entries + row_cost * its rows (row_cost 0:
    equal entries)."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    n = row_ptr.shape[0] - 1
    cost = row_ptr.astype(np.float64) + float(row_cost) * np.arange(n + 1, dtype=np.float64)
    total = float(cost[-1])
    targets = [total * r / world for r in range(1, world)]
    inner = [int(np.searchsorted(cost, t, side="left")) for t in targets]
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
    ws, wsb = native_ops._workspace(dev, N.lib().gnn_spmm_schedule_workspace_bytes(shard.num_rows, shard.num_edges))
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
    """Where every global row lives in the padded [chunks*world*Mc, F] exchange matrix.

    Rank r owns the rows order[r] (global ids, increasing) in that local order.
    Its local rows are cut into `chunks` pieces of `chunk_rows` (Mc) rows, and
    local row i of rank r lives at padded id

        (i // Mc) * world * Mc  +  r * Mc  +  (i % Mc)

    so piece c of every rank forms the contiguous block [c*world*Mc,
    (c+1)*world*Mc) of the padded matrix: exchanging piece c is one
    all_gather_into_tensor (or one push per peer) straight into the next
    layer's input while piece c+1 is still being computed. Padding rows are
    never referenced by any column id. The renumbering only rewrites column
    values; CSR entry order, and therefore every floating-point sum, is
    unchanged. With one rank's rows a contiguous range and chunks == 1 this is
    the plain layout r*Mc + i.

    rank_major=True places local row i of rank r at r * chunks * Mc + i
    instead: every rank's rows form one contiguous block (a layer can then run
    as one call over all of them) and piece c is [Mc] rows inside it. The
    peer-to-peer exchanges (push, halo) work with either; the all_gather
    exchange needs the chunk-major order.
    """
    order: list[torch.Tensor]
    chunk_rows: int
    chunks: int = 1
    rank_major: bool = False

    def __post_init__(self):
        self.order = [torch.as_tensor(o, dtype=torch.int64).cpu().contiguous() for o in self.order]
        n = sum(int(o.numel()) for o in self.order)
        ids = torch.full((n,), -1, dtype=torch.int64)
        mc, w = self.chunk_rows, self.world
        for r, o in enumerate(self.order):
            i = torch.arange(o.numel(), dtype=torch.int64)
            if self.rank_major:
                ids[o] = r * self.chunks * mc + i
            else:
                ids[o] = (i // mc) * (w * mc) + r * mc + (i % mc)
        if n and int(ids.min()) < 0:
            raise ValueError("the rank orders must cover every row exactly once")
        self.ids = ids
        self._ids_on: dict = {}

    @property
    def world(self) -> int:
        return len(self.order)

    @property
    def num_nodes(self) -> int:
        return int(self.ids.numel())

    @property
    def local_rows(self) -> int:
        """Rows of one rank's padded output buffer (chunks * Mc)."""
        return self.chunks * self.chunk_rows

    @property
    def padded_rows(self) -> int:
        return self.chunks * self.world * self.chunk_rows

    def rows_of(self, rank: int) -> int:
        return int(self.order[rank].numel())

    def piece_range(self, rank: int, c: int) -> tuple[int, int]:
        """Local row range [lo, hi) of piece c on `rank` (possibly empty)."""
        lo = min(c * self.chunk_rows, self.rows_of(rank))
        return lo, min((c + 1) * self.chunk_rows, self.rows_of(rank))

    def piece_first(self, rank: int, c: int) -> int:
        """Padded id of piece c's first row on `rank`."""
        if self.rank_major:
            return (rank * self.chunks + c) * self.chunk_rows
        return c * self.world * self.chunk_rows + rank * self.chunk_rows

    def piece_of(self, padded: torch.Tensor) -> torch.Tensor:
        """Piece index of each padded row id."""
        if self.rank_major:
            return (padded % (self.chunks * self.chunk_rows)) // self.chunk_rows
        return padded // (self.world * self.chunk_rows)

    def contiguous_ranks(self) -> bool:
        """Every rank's rows are one contiguous block of padded ids."""
        return self.rank_major or self.chunks == 1

    def ids_on(self, device) -> torch.Tensor:
        key = str(device)
        if key not in self._ids_on:
            self._ids_on[key] = self.ids.to(device)
        return self._ids_on[key]

    def padded_ids(self, g: torch.Tensor) -> torch.Tensor:
        return self.ids_on(g.device)[g.to(torch.int64)]

    def pad_rows(self, full: torch.Tensor) -> torch.Tensor:
        """[N, ...] -> [padded_rows, ...] with zero padding rows."""
        out = torch.zeros((self.padded_rows,) + tuple(full.shape[1:]), dtype=full.dtype, device=full.device)
        out[self.ids_on(full.device)] = full
        return out

    def unpad_rows(self, padded: torch.Tensor) -> torch.Tensor:
        return padded[self.ids_on(padded.device)]


def balanced_row_order(row_ptr: np.ndarray, world: int, row_cost: float = ROW_COST_IN_ENTRIES) -> list[np.ndarray]:
    """Deal rows to ranks so that every rank gets the same number of rows (+-1)
    and about the same cost (entries + row_cost per row): rows sorted by cost,
    heaviest first, are dealt 0, 1, .., W-1, W-1, .., 0, 0, 1, ... Each rank then
    keeps its rows in increasing id order. Power-law hubs end up spread over all
    ranks instead of packed into the first one, so neither the aggregation nor
    the exchange (each rank sends its rows to every peer) is dominated by one rank."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    n = rp.shape[0] - 1
    cost = np.diff(rp).astype(np.float64) + float(row_cost)
    by_cost = np.argsort(-cost, kind="stable")
    p = np.arange(n)
    w = p % world
    owner = np.empty(n, dtype=np.int64)
    owner[by_cost] = np.where((p // world) % 2 == 0, w, world - 1 - w)
    return [np.nonzero(owner == r)[0] for r in range(world)]


def make_padded_layout(row_ptr: np.ndarray, world: int, chunks: int = 1, *, balanced: bool = False,
                       row_cost: float = 0.0, rank_major: bool = False) -> PaddedLayout:
    """Contiguous cost-balanced row ranges (balanced=False), or rows dealt by
    balanced_row_order (balanced=True), in `chunks` pieces per rank, placed
    chunk-major or rank-major (PaddedLayout)."""
    if balanced:
        order = balanced_row_order(row_ptr, world, row_cost)
    else:
        bounds = nnz_balanced_bounds(row_ptr, world, row_cost)
        order = [np.arange(bounds[r], bounds[r + 1]) for r in range(world)]
    max_rows = max(1, max(len(o) for o in order))
    chunks = max(1, min(int(chunks), max_rows))
    return PaddedLayout(order, -(-max_rows // chunks), chunks, rank_major)


@dataclass
class PaddedShard:
    """One rank's rows as `chunks` row pieces with padded row and column ids."""
    rank: int
    pieces: list[RowShard]  # piece c: row_begin = its first padded row (also the dis lookup)
    whole: RowShard | None = None  # all rows as one shard, when they are contiguous padded ids

    @property
    def num_rows(self) -> int:
        return sum(p.num_rows for p in self.pieces)

    @property
    def num_edges(self) -> int:
        return sum(p.num_edges for p in self.pieces)

    def device_tensors(self) -> list[torch.Tensor]:
        """The distinct device tensors holding this shard (the pieces' column ids
        are views of the whole shard's when it exists)."""
        ts = [p.row_ptr for p in self.pieces if p.num_rows]
        if self.whole is not None:
            return ts + [self.whole.row_ptr, self.whole.col_ind]
        return ts + [p.col_ind for p in self.pieces if p.num_edges]


def make_padded_shard(row_ptr: torch.Tensor, col_ind: torch.Tensor, layout: PaddedLayout, rank: int) -> PaddedShard:
    """Rank `rank`'s rows (layout.order[rank]) gathered into their own CSR, cut into
    the layout's pieces, column ids rewritten to padded ids. Entry order within
    every row is kept."""
    dev = row_ptr.device
    rows = layout.order[rank].to(dev)
    rp64 = row_ptr.to(torch.int64)
    starts = rp64[rows]
    deg = rp64[rows + 1] - starts
    local_rp = torch.zeros(rows.numel() + 1, dtype=torch.int64, device=dev)
    torch.cumsum(deg, 0, out=local_rp[1:])
    total = int(local_rp[-1])
    first, last = (int(rows[0]), int(rows[-1])) if rows.numel() else (0, -1)
    if rows.numel() and last - first + 1 == rows.numel():  # a contiguous range: a slice
        e0 = int(rp64[first])
        cols_g = col_ind[e0:e0 + total]
    else:
        entry = starts.repeat_interleave(deg) + (torch.arange(total, device=dev) - local_rp[:-1].repeat_interleave(deg))
        cols_g = col_ind[entry]
    cols = layout.padded_ids(cols_g).to(torch.int32) if total else col_ind[:0].to(torch.int32)
    pieces = []
    for c in range(layout.chunks):
        lo, hi = layout.piece_range(rank, c)
        e0, e1 = int(local_rp[lo]), int(local_rp[hi])
        rp_c = (local_rp[lo:hi + 1] - e0).to(row_ptr.dtype).contiguous()
        head = layout.piece_first(rank, c)
        pieces.append(RowShard(head, head + (hi - lo), rp_c, cols[e0:e1]))  # a view of cols
    whole = None
    if layout.contiguous_ranks():
        head = layout.piece_first(rank, 0)
        whole = RowShard(head, head + int(rows.numel()), local_rp.to(row_ptr.dtype).contiguous(), cols)
    return PaddedShard(rank, pieces, whole)


@dataclass
class HaloPlan:
    """The rows of one rank that its peers read, per row piece: the halo push list.

    For piece c, ``ids[c]`` (int32, device) holds padded row ids of this rank's
    piece c, grouped by peer in ``peers`` order and sorted within a group;
    peer ``peers[q]`` receives ids[c][offsets[c][q]:offsets[c][q+1]]. A peer
    reads a remote row only through a column id of its CSR, so these are
    exactly the rows it needs; the rest of its copy of the next layer's input
    is never read and need not be sent.
    """
    rank: int
    peers: list[int]
    ids: list[torch.Tensor]
    offsets: list[list[int]]

    @property
    def rows_sent(self) -> int:
        return sum(o[-1] for o in self.offsets)

    def piece_masks(self, shard: "PaddedShard") -> list[torch.Tensor]:
        """The same lists as one byte per row of each piece (uint8, on the ids'
        device): bit q of row i is set when peers[q] reads row i of the piece.
        This is the form the transform's fused push reads (gnn_linear_push_forward)."""
        if self.peers and len(self.peers) > 8:
            raise ValueError("a row mask holds at most 8 peers")
        masks = []
        for c, piece in enumerate(shard.pieces):
            ids = self.ids[c]
            m = torch.zeros(piece.num_rows, dtype=torch.uint8, device=ids.device)
            off = self.offsets[c]
            for q in range(len(self.peers)):
                seg = ids[off[q]:off[q + 1]].to(torch.int64) - piece.row_begin
                if seg.numel():
                    m[seg] |= 1 << q
            masks.append(m)
        return masks


def make_halo_plan(row_ptr: torch.Tensor, col_ind: torch.Tensor, layout: PaddedLayout, rank: int) -> HaloPlan:
    """Halo lists of `rank` from the global CSR (global ids, any device): every
    (peer, column) pair where a row owned by the peer reads a column owned by
    `rank`, de-duplicated, as padded ids split by `rank`'s row pieces."""
    dev = row_ptr.device
    n, w = layout.num_nodes, layout.world
    owner = torch.empty(n, dtype=torch.int64, device=dev)
    for r, o in enumerate(layout.order):
        owner[o.to(dev)] = r
    rp64 = row_ptr.to(torch.int64)
    row_owner = owner.repeat_interleave(rp64[1:] - rp64[:-1])
    col = col_ind.to(torch.int64)
    sel = (owner[col] == rank) & (row_owner != rank)
    pid = layout.padded_ids(col[sel])
    total_rows = layout.padded_rows
    key = torch.unique(row_owner[sel] * total_rows + pid)  # peer-major, then padded id
    del owner, row_owner, col, sel, pid
    peer_of = key // total_rows
    ids = key - peer_of * total_rows
    piece = layout.piece_of(ids)
    peers = [p for p in range(w) if p != rank]
    out_ids, out_off = [], []
    for c in range(layout.chunks):
        m = piece == c
        ids_c, peer_c = ids[m], peer_of[m]
        counts = torch.bincount(peer_c, minlength=w).cpu().tolist() if peer_c.numel() else [0] * w
        off = [0]
        for p in peers:
            off.append(off[-1] + int(counts[p]))
        out_ids.append(ids_c.to(torch.int32).contiguous())
        out_off.append(off)
    return HaloPlan(rank, peers, out_ids, out_off)


def allgather_buffers(layout: PaddedLayout, feat: int, device) -> dict:
    """Buffers for gcn_forward_allgather: 'agg' [Mc, F], 'out' [chunks*Mc, F]
    (padding rows zero), 'x_next' [padded_rows, F]."""
    return {"agg": torch.empty(layout.chunk_rows, feat, device=device),
            "out": torch.zeros(layout.local_rows, feat, device=device),
            "x_next": torch.empty(layout.padded_rows, feat, device=device)}


def gcn_forward_allgather(shard: PaddedShard, dis_pad: torch.Tensor, x_pad: torch.Tensor, weights: list[torch.Tensor],
                          biases: list[torch.Tensor], layout: PaddedLayout, bufs: dict, group=None,
                          timers: dict | None = None) -> torch.Tensor:
    """Multi-layer GCN over a padded-layout shard, exchange pipelined by row piece.

    For each piece c: aggregation, X·W + b (+ReLU) into out[c*Mc:...], then an
    asynchronous all_gather of that piece on the collective stream while the
    compute stream goes on with piece c+1. The next layer waits for all
    pieces. Returns this rank's [rows, F] output rows (local order).
    """
    if layout.rank_major and layout.chunks > 1:
        raise ValueError("the all_gather exchange needs the chunk-major layout")
    x = x_pad
    layers = len(weights)
    mc, world = layout.chunk_rows, layout.world
    out = bufs["out"]
    for li in range(layers):
        last = li == layers - 1
        works = []
        for c, piece in enumerate(shard.pieces):
            lo = c * mc
            rows_c = piece.num_rows
            if rows_c:
                agg = bufs["agg"][:rows_c]
                ev = _mark(timers, "spmm_begin")
                spmm_gcn_shard(piece, dis_pad, x, agg)
                _mark(timers, "spmm_end", ev)
                native_ops.linear_forward_(agg, weights[li], biases[li], out[lo:lo + rows_c], not last)
            if not last:
                works.append(dist.all_gather_into_tensor(bufs["x_next"][c * world * mc:(c + 1) * world * mc],
                                                         out[lo:lo + mc], group=group, async_op=True))
        if last:
            break
        for w in works:
            w.wait()
        x = bufs["x_next"]
    return out[:shard.num_rows]


def piece_bounds(row_ptr: np.ndarray, chunks: int) -> list[int]:
    """Local row boundaries cutting a shard into at most `chunks` non-empty pieces of about equal nnz."""
    n = int(np.asarray(row_ptr).shape[0]) - 1
    b = nnz_balanced_bounds(row_ptr, max(1, min(int(chunks), max(n, 1))))
    out = [b[0]]
    for v in b[1:]:
        if v > out[-1]:
            out.append(v)
    if len(out) == 1:
        out.append(n)
    return out


def make_pieces(row_ptr: torch.Tensor, col_ind: torch.Tensor, row_begin: int, row_end: int,
                chunks: int) -> list[RowShard]:
    """Rows [row_begin, row_end) as equal-nnz RowShards with global row and column ids."""
    rp = row_ptr[row_begin:row_end + 1].to(torch.int64).cpu().numpy()
    b = piece_bounds(rp - rp[0], chunks)
    return [make_shard(row_ptr, col_ind, row_begin + lo, row_begin + hi) for lo, hi in zip(b[:-1], b[1:])]


class _PeerBlock:
    """Owner of a gnn_peer_alloc buffer exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, device: int):
        self.ptr, self.device = ptr, device
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": "<f4",
                                         "data": (ptr, False), "version": 3, "strides": None}

    def free(self):
        if self.ptr:
            N.call("gnn_peer_free", ctypes.c_void_p(self.ptr), self.device)
            self.ptr = 0


class PeerRowExchange:
    """Row exchange between the ranks of one node through IPC-mapped peer buffers.

    Every rank holds two [rows, F] copies of "the next layer's input" in memory
    it allocated itself (gnn_peer_alloc) and has mapped every peer's copies
    through CUDA IPC. A layer writes its output rows straight into the rank's
    own rows of the current copy; `push` sends a finished row range to the same
    rows of every peer's current copy once an event has fired:
      * transport "sm": one gnn_peer_push kernel on the push stream reads the
        rows once and stores them to all peers (SMs drive NVLink; `ctas` bounds
        its grid so that it can share the GPU with the next piece's aggregation);
      * transport "ce": one cudaMemcpyAsync per peer on that peer's stream
        (copy engines, no SM).
    `finish` is the device-side barrier: a one-element NCCL all_reduce issued
    after every push, which the compute stream waits on before reading the copy.
    Copies alternate per exchange, so a push never lands in a copy that a peer
    can still be reading: a rank pushes into copy t only after the barrier of
    the previous exchange, which every peer reaches only after its last read of
    copy t.
    """

    def __init__(self, num_rows: int, feat: int, rank: int, world: int, device: torch.device, group=None,
                 transport: str = "sm", ctas: int = 0):
        if transport not in ("sm", "ce"):
            raise ValueError("transport must be 'sm' or 'ce'")
        if world - 1 > 8 and transport == "sm":
            raise ValueError("the sm transport pushes to at most 8 peers")
        self.rank, self.world, self.group = rank, world, group
        self.transport, self.ctas = transport, int(ctas)
        self.device = device
        self.row_bytes = feat * 4
        self.shape = (num_rows, feat)
        dev = device.index
        nbytes = max(1, num_rows * feat * 4)
        self._blocks, self.buffers, handles = [], [], []
        hb = int(N.lib().gnn_ipc_handle_bytes())
        for _ in range(2):
            p = ctypes.c_void_p(0)
            N.call("gnn_peer_alloc", nbytes, dev, ctypes.byref(p))
            blk = _PeerBlock(p.value, self.shape, dev)
            self._blocks.append(blk)
            with torch.cuda.device(dev):
                self.buffers.append(torch.as_tensor(blk, device=device))
            h = ctypes.create_string_buffer(hb)
            N.call("gnn_ipc_get_handle", ctypes.c_void_p(p.value), h, hb)
            handles.append(h.raw)
        everyone: list = [None] * world
        dist.all_gather_object(everyone, handles, group=group)
        # peer_ptrs[t][p]: peer p's copy t, mapped here
        self.peer_ptrs: list[dict[int, int]] = [{}, {}]
        for p in range(world):
            if p == rank:
                continue
            for t in range(2):
                ptr = ctypes.c_void_p(0)
                buf = ctypes.create_string_buffer(everyone[p][t], hb)
                N.call("gnn_ipc_open", buf, hb, dev, ctypes.byref(ptr))
                self.peer_ptrs[t][p] = ptr.value
        if transport == "ce":
            self.streams = {p: torch.cuda.Stream(device) for p in self.peer_ptrs[0]}
        else:
            self.streams = {-1: torch.cuda.Stream(device)}
        self.barrier_stream = torch.cuda.Stream(device)
        self.flag = torch.zeros(1, device=device)
        self.turn = 0

    def buffer(self) -> torch.Tensor:
        """The copy that the current exchange fills."""
        return self.buffers[self.turn]

    def push(self, row_lo: int, row_hi: int, ready: torch.cuda.Event) -> None:
        """Send rows [row_lo, row_hi) of the current copy to every peer once `ready` has fired."""
        if row_hi <= row_lo or not self.peer_ptrs[self.turn]:
            return
        off = row_lo * self.row_bytes
        nbytes = (row_hi - row_lo) * self.row_bytes
        src = self.buffers[self.turn].data_ptr() + off
        if self.transport == "sm":
            s = self.streams[-1]
            s.wait_event(ready)
            dsts = [ptr + off for ptr in self.peer_ptrs[self.turn].values()]
            arr = (ctypes.c_void_p * len(dsts))(*dsts)
            N.call("gnn_peer_push", ctypes.c_void_p(src), arr, len(dsts), nbytes, self.ctas,
                   ctypes.c_void_p(s.cuda_stream))
            return
        for p, s in self.streams.items():
            s.wait_event(ready)
            N.call("gnn_copy_async", ctypes.c_void_p(self.peer_ptrs[self.turn][p] + off), ctypes.c_void_p(src),
                   nbytes, ctypes.c_void_p(s.cuda_stream))

    def push_rows(self, ids: torch.Tensor, offsets: list[int], peers: list[int], ready: torch.cuda.Event) -> None:
        """Halo push: send the listed rows of the current copy (ids[offsets[q]:offsets[q+1]]
        to peers[q]) once `ready` has fired; one gnn_peer_push_rows kernel on the push stream."""
        if offsets[-1] == 0 or not self.peer_ptrs[self.turn]:
            return
        if self.transport != "sm":
            raise ValueError("halo pushes need the sm transport")
        s = self.streams[-1]
        s.wait_event(ready)
        dsts = [self.peer_ptrs[self.turn][p] for p in peers]
        arr = (ctypes.c_void_p * len(dsts))(*dsts)
        offs = (ctypes.c_int64 * len(offsets))(*offsets)
        N.call("gnn_peer_push_rows", ctypes.c_void_p(self.buffers[self.turn].data_ptr()), arr, len(dsts),
               ctypes.c_void_p(ids.data_ptr()), offs, self.row_bytes, self.shape[0], self.ctas,
               ctypes.c_void_p(s.cuda_stream))

    def peer_rows(self, row_begin: int, peers: list[int]) -> list[int]:
        """Device addresses of row `row_begin` of each peer's current copy (in `peers`
        order), for a kernel on the compute stream that stores rows to the peers
        itself (the fused push of the transform)."""
        return [self.peer_ptrs[self.turn][p] + row_begin * self.row_bytes for p in peers]

    def finish(self) -> torch.Tensor:
        """Barrier after every rank's pushes; returns the completed copy and moves to the other one.

        The barrier also follows the work issued so far on the calling stream, where a
        fused push (rows stored to the peers by the transform itself) runs."""
        for s in self.streams.values():
            self.barrier_stream.wait_stream(s)
        self.barrier_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.barrier_stream):
            work = dist.all_reduce(self.flag, group=self.group, async_op=True)
        work.wait()  # the current (compute) stream waits for the barrier
        done = self.buffers[self.turn]
        self.turn ^= 1
        return done

    def close(self) -> None:
        """Unmap the peers' copies, then free this rank's copies (all ranks call this)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for t in range(2):
            for p, ptr in self.peer_ptrs[t].items():
                N.call("gnn_ipc_close", ctypes.c_void_p(ptr), self.device.index)
            self.peer_ptrs[t] = {}
        dist.barrier(group=self.group)
        self.buffers = []
        for blk in self._blocks:
            blk.free()
        self._blocks = []


def gcn_forward_push(shard: PaddedShard, dis_pad: torch.Tensor, x_pad: torch.Tensor, weights: list[torch.Tensor],
                     biases: list[torch.Tensor], layout: PaddedLayout, exchange: PeerRowExchange, agg: torch.Tensor,
                     out: torch.Tensor, timers: dict | None = None, halo: HaloPlan | None = None,
                     trace: list | None = None, push_masks: list[torch.Tensor] | None = None) -> torch.Tensor:
    """Multi-layer GCN over a padded-layout shard; layer outputs pushed to the peers piece by piece.

    exchange: a PeerRowExchange over layout.padded_rows rows. agg: [Mc, F]
    scratch, or [chunks*Mc, F]. out: [chunks*Mc, F] for the last layer (local
    order). Each piece's aggregation and X·W + b (+ReLU) land in this rank's
    rows of the exchange's current copy, which are then pushed to the peers
    while the next piece is computed. With a `halo` plan only the rows each peer
    reads are pushed. The last layer pushes nothing, so when the shard's rows
    are one contiguous block (shard.whole) and agg holds them all it runs as
    one aggregation call and one transform: the same per-row sums as the
    pieces, without a call per piece. With `push_masks` (halo.piece_masks(shard))
    the transform stores the halo rows to the peers itself, from its epilogue
    while later tiles are computed (gnn_linear_push_forward), instead of a push
    kernel after it; where that kernel does not apply the separate push runs.
    Returns this rank's [rows, F] output rows (local order). With `trace`, a list,
    (label, event) pairs are appended for one step's timeline: the start, every
    piece's aggregation and transform end (compute stream), its push end (push
    stream) and the end of the wait for the exchange.
    """
    layers = len(weights)
    mc = layout.chunk_rows
    h = x_pad
    _trace(trace, "start")
    whole_last = shard.whole is not None and shard.whole.num_rows <= agg.size(0) and len(shard.pieces) > 1
    for li in range(layers):
        last = li == layers - 1
        pieces = [shard.whole] if last and whole_last else shard.pieces
        for c, piece in enumerate(pieces):
            if piece.num_rows == 0:
                continue
            a = agg[:piece.num_rows]
            ev = _mark(timers, "spmm_begin")
            t0 = _host_clock(timers)
            spmm_gcn_shard(piece, dis_pad, h, a)
            t0 = _host_time(timers, "aggregate", t0)
            _mark(timers, "spmm_end", ev)
            _trace(trace, f"l{li}p{c}_agg")
            if last:
                dst = out[c * mc:c * mc + piece.num_rows]
            else:
                dst = exchange.buffer()[piece.row_begin:piece.row_end]
            fused = (not last and push_masks is not None and halo is not None and exchange.transport == "sm" and
                     native_ops.linear_push_forward_(a, weights[li], biases[li], dst, True, push_masks[c],
                                                     exchange.peer_rows(piece.row_begin, halo.peers)))
            if not fused:
                native_ops.linear_forward_(a, weights[li], biases[li], dst, not last)
            t0 = _host_time(timers, "transform", t0)
            _trace(trace, f"l{li}p{c}_gemm")
            if not last and not fused:
                ready = torch.cuda.Event()
                ready.record()
                if halo is None:
                    exchange.push(piece.row_begin, piece.row_end, ready)
                else:
                    exchange.push_rows(halo.ids[c], halo.offsets[c], halo.peers, ready)
                _host_time(timers, "push", t0)
                for s in exchange.streams.values():
                    _trace(trace, f"l{li}p{c}_push", s)
        if not last:
            ev = _mark(timers, "xchg_begin")
            t0 = _host_clock(timers)
            h = exchange.finish()
            _host_time(timers, "barrier", t0)
            _mark(timers, "xchg_end", ev, series="xchg")
            _trace(trace, f"l{li}_exchanged")
    return out[:shard.num_rows]


class PushForwardGraphs:
    """One step of gcn_forward_push (any callable that runs one) captured as CUDA
    graphs, so that a step is issued by one launch.

    Issued from Python a step is dozens of launches, events and a collective; on
    8 GPUs a rank's step is about 2 ms of device work and the host issued it more
    slowly than that. Every finish() moves the exchange to its other copy, so two
    consecutive steps are captured (one per copy) and replayed in the order the
    copies take; replay() advances exchange.turn exactly as an eager step does,
    so eager steps and replays can follow one another. Every rank must capture
    and replay the same steps in the same order (the barrier collective is part
    of each graph). Call close() before the process group is destroyed.
    """

    def __init__(self, step_fn, exchange: "PeerRowExchange"):
        self.exchange = exchange
        self.first_turn = exchange.turn
        self.graphs = []
        self.out = None
        try:
            for _ in range(2):
                before = exchange.turn
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    self.out = step_fn()
                self.graphs.append(g)
                if exchange.turn != before ^ 1:
                    raise RuntimeError("a captured step must finish exactly one exchange")
        except Exception:
            # every rank must go on from the same copy, whether its capture failed or not
            exchange.turn = self.first_turn
            self.graphs = []
            raise

    def replay(self) -> torch.Tensor:
        self.graphs[self.exchange.turn ^ self.first_turn].replay()
        self.exchange.turn ^= 1
        return self.out

    def close(self) -> None:
        self.graphs = []


def _host_clock(timers: dict | None) -> float:
    return time.perf_counter() if timers is not None else 0.0


def _host_time(timers: dict | None, key: str, t0: float) -> float:
    """Add the host time since t0 to timers["host"][key] (seconds); returns now."""
    if timers is None:
        return 0.0
    now = time.perf_counter()
    host = timers.setdefault("host", {})
    host[key] = host.get(key, 0.0) + (now - t0)
    return now


def _trace(trace: list | None, label: str, stream=None) -> None:
    """Append (label, timing event recorded on `stream` or the current stream)."""
    if trace is None:
        return
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(stream)
    trace.append((label, ev))


def trace_offsets(trace: list) -> dict:
    """{label: ms after the first event} of a synchronised trace (the last event of a label wins)."""
    t0 = trace[0][1]
    return {label: round(t0.elapsed_time(ev), 4) for label, ev in trace}


def _mark(timers: dict | None, key: str, begin=None, *, series: str = "spmm"):
    """Record a CUDA event on the current stream for per-phase timing.

    With `begin`, the (begin, end) pair is appended to timers[series] ("spmm":
    one entry per aggregation piece; "xchg": the wait for a layer-boundary
    exchange to complete, as the compute stream sees it)."""
    if timers is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    if begin is not None:
        timers.setdefault(series, []).append((begin, ev))
    return ev
