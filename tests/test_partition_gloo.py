"""Row partitioning and the between-layer row exchange, as world-size-2 gloo ranks on CPU.

The CUDA aggregation is replaced here by the oracle (CPU test only): the test
covers the host logic of the multi-GPU mode — equal-nnz bounds, shard
construction with global column ids, the broadcast-based exchange and the
padded chunk-major layout with its pipelined all_gather — and checks that the
exchanged outputs equal the single-rank result bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gnn_cuda_b200 import partition, synth


def test_bounds_balance_nnz():
    u, v = synth.rmat_undirected(5000, 40000, seed=2)
    s, d = synth.symmetrize(u, v)
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    g = G.build_gcn_normalized_csr(s, d, num_nodes=5000)
    rp = g.row_ptr.numpy().astype(np.int64)
    for world in (1, 2, 3, 4, 8):
        b = partition.nnz_balanced_bounds(rp, world)
        assert b[0] == 0 and b[-1] == 5000 and all(b[i] <= b[i + 1] for i in range(world))
        loads = [rp[b[i + 1]] - rp[b[i]] for i in range(world)]
        assert max(loads) - min(loads) <= rp[1:].max() - rp[:-1].min() + np.diff(rp).max() * 2
    # with a per-row cost, ranges balance entries + row_cost * rows
    for world in (2, 4, 8):
        b = partition.nnz_balanced_bounds(rp, world, row_cost=6)
        costs = [rp[b[i + 1]] - rp[b[i]] + 6 * (b[i + 1] - b[i]) for i in range(world)]
        assert b[0] == 0 and b[-1] == 5000 and b == sorted(b)
        assert max(costs) - min(costs) <= 2 * (np.diff(rp).max() + 6)
    # one giant row heavier than a share keeps bounds monotone
    rp2 = np.array([0, 1000, 1001, 1002, 1003], dtype=np.int64)
    b = partition.nnz_balanced_bounds(rp2, 4)
    assert b[0] == 0 and b[-1] == 4 and b == sorted(b)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
        n, f = 1200, 16
        u, v = synth.rmat_undirected(n, 9000, seed=5)
        s, d = synth.symmetrize(u, v)
        g = G.build_gcn_normalized_csr(s, d, num_nodes=n)
        x = synth.features(n, f, seed=6)
        bounds = partition.nnz_balanced_bounds(g.row_ptr.numpy(), world)
        shard = partition.make_shard(g.row_ptr, g.col_ind, bounds[rank], bounds[rank + 1])
        # layer 1 on this shard's rows (oracle aggregation with global column ids)
        rp_local = shard.row_ptr.numpy()
        dis = g.deg_inv_sqrt.numpy()
        # weight rows by dis[global row] * dis[col] through the edge-weight path
        rows = np.repeat(np.arange(shard.num_rows) + shard.row_begin, np.diff(rp_local))
        ew = (dis[rows] * dis[shard.col_ind.numpy()]).astype(np.float32)
        out = O.spmm(rp_local, shard.col_ind.numpy(), x.numpy(), mode=O.W_EDGE, ew=ew)
        full = torch.empty(n, f)
        partition.exchange_rows(torch.from_numpy(out), full, bounds, rank)
        q.put((rank, full.numpy()))
    finally:
        dist.destroy_process_group()


def test_piece_bounds_and_pieces():
    rp = np.array([0, 10, 10, 10, 11, 30], dtype=np.int64)
    for chunks in (1, 2, 3, 5, 9):
        b = partition.piece_bounds(rp, chunks)
        assert b[0] == 0 and b[-1] == 5 and all(b[i] < b[i + 1] for i in range(len(b) - 1))
        assert len(b) - 1 <= chunks
    assert partition.piece_bounds(np.array([0]), 4) == [0, 0]  # no rows: one empty piece
    u, v = synth.rmat_undirected(700, 5000, seed=3)
    s, d = synth.symmetrize(u, v)
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    g = G.build_gcn_normalized_csr(s, d, num_nodes=700)
    pieces = partition.make_pieces(g.row_ptr, g.col_ind, 100, 650, 4)
    assert pieces[0].row_begin == 100 and pieces[-1].row_end == 650
    assert all(a.row_end == b.row_begin for a, b in zip(pieces[:-1], pieces[1:]))
    cols = torch.cat([p.col_ind for p in pieces])
    assert torch.equal(cols, g.col_ind[g.row_ptr[100]:g.row_ptr[650]])  # global ids, CSR order kept
    for p in pieces:
        assert int(p.row_ptr[0]) == 0 and int(p.row_ptr[-1]) == p.num_edges


def test_padded_layout_maps():
    rp = np.array([0, 3, 3, 10, 12, 20, 21, 30], dtype=np.int64)  # 7 rows
    lay = partition.make_padded_layout(rp, 3)
    assert lay.world == 3 and lay.num_nodes == 7
    assert [int(o[0]) for o in lay.order if o.numel()] == sorted(int(o[0]) for o in lay.order if o.numel())
    g = torch.arange(7)
    p = lay.padded_ids(g)
    assert torch.all(p[1:] > p[:-1])  # contiguous ranges, one piece: the plain r*Mc + i layout, increasing
    x = torch.arange(7 * 2, dtype=torch.float32).view(7, 2)
    xp = lay.pad_rows(x)
    assert xp.shape == (lay.padded_rows, 2)
    assert torch.equal(xp[p], x) and torch.equal(lay.unpad_rows(xp), x)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_balanced_row_order(world):
    u, v = synth.rmat_undirected(4000, 40000, seed=world)
    s, d = synth.symmetrize(u, v)
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    rp = G.build_gcn_normalized_csr(s, d, num_nodes=4000).row_ptr.numpy().astype(np.int64)
    order = partition.balanced_row_order(rp, world, row_cost=6)
    allrows = np.sort(np.concatenate(order))
    assert np.array_equal(allrows, np.arange(4000))  # every row exactly once
    sizes = [len(o) for o in order]
    assert max(sizes) - min(sizes) <= 1  # equal rows per rank
    deg = np.diff(rp)
    costs = [float((deg[o] + 6).sum()) for o in order]
    assert max(costs) - min(costs) <= deg.max() + 6  # the snake deal keeps costs within one row
    assert all(np.all(np.diff(o) > 0) for o in order)  # increasing ids within a rank


@pytest.mark.parametrize("rank_major", [False, True])
@pytest.mark.parametrize("world,chunks,balanced", [(2, 3, False), (3, 2, False), (4, 5, True), (2, 64, True),
                                                   (3, 1, True)])
def test_padded_layout_pieces(world, chunks, balanced, rank_major):
    u, v = synth.rmat_undirected(300, 2000, seed=world + chunks)
    s, d = synth.symmetrize(u, v)
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    g = G.build_gcn_normalized_csr(s, d, num_nodes=300)
    lay = partition.make_padded_layout(g.row_ptr.numpy(), world, chunks, balanced=balanced, row_cost=6,
                                       rank_major=rank_major)
    ids = lay.padded_ids(torch.arange(300))
    assert len(set(ids.tolist())) == 300 and int(ids.max()) < lay.padded_rows  # injective, in range
    mc = lay.chunk_rows
    for r in range(world):
        rows = lay.order[r]
        for c in range(lay.chunks):
            lo, hi = lay.piece_range(r, c)
            got = ids[rows[lo:hi]]
            want = lay.piece_first(r, c) + torch.arange(hi - lo)
            assert torch.equal(got, want)  # piece c of rank r is one contiguous block
            assert bool((lay.piece_of(got) == c).all())
        if lay.contiguous_ranks():  # all of rank r's rows are one block
            assert torch.equal(ids[rows], lay.piece_first(r, 0) + torch.arange(rows.numel()))
    # the shard holds exactly its rows' entries, in CSR order, renumbered
    rp = g.row_ptr.to(torch.int64)
    for r in range(world):
        sh = partition.make_padded_shard(g.row_ptr, g.col_ind, lay, r)
        rows = lay.order[r]
        want_cols = torch.cat([g.col_ind[rp[v]:rp[v + 1]] for v in rows.tolist()] or [g.col_ind[:0]])
        assert sh.num_rows == rows.numel() and sh.num_edges == want_cols.numel()
        cols = torch.cat([p.col_ind.to(torch.int64) for p in sh.pieces])
        assert torch.equal(cols, ids[want_cols.to(torch.int64)])
        for c, p in enumerate(sh.pieces):
            lo, hi = lay.piece_range(r, c)
            assert p.row_begin == lay.piece_first(r, c) and p.num_rows == hi - lo
            seg = rows[lo:hi]
            assert int(p.row_ptr[0]) == 0
            assert torch.equal(torch.diff(p.row_ptr.to(torch.int64)), rp[seg + 1] - rp[seg])  # row degrees
        assert (sh.whole is not None) == lay.contiguous_ranks()
        if sh.whole is not None:  # the whole shard is the pieces laid end to end
            assert sh.whole.row_begin == lay.piece_first(r, 0) and sh.whole.num_rows == rows.numel()
            assert torch.equal(sh.whole.col_ind.to(torch.int64), cols)
            assert torch.equal(torch.diff(sh.whole.row_ptr.to(torch.int64)), rp[rows + 1] - rp[rows])
    x = torch.randn(300, 3)
    assert torch.equal(lay.unpad_rows(lay.pad_rows(x)), x)


def _worker_padded(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
        n, f = 1500, 8
        u, v = synth.rmat_undirected(n, 11000, seed=7)
        s, d = synth.symmetrize(u, v)
        g = G.build_gcn_normalized_csr(s, d, num_nodes=n)
        x = synth.features(n, f, seed=8)
        results = []
        for chunks, balanced in ((1, False), (4, False), (1, True), (3, True)):
            lay = partition.make_padded_layout(g.row_ptr.numpy(), world, chunks, balanced=balanced, row_cost=6)
            shard = partition.make_padded_shard(g.row_ptr, g.col_ind, lay, rank)
            dis_pad = lay.pad_rows(g.deg_inv_sqrt).numpy()
            x_pad = lay.pad_rows(x).numpy()
            out = torch.zeros(lay.local_rows, f)
            gathered = torch.empty(lay.padded_rows, f)
            works = []
            mc = lay.chunk_rows
            # per piece: aggregate its rows (oracle, CPU test only), then start its exchange
            for c, piece in enumerate(shard.pieces):
                if piece.num_rows:
                    rp_local = piece.row_ptr.numpy()
                    rows = np.repeat(np.arange(piece.num_rows) + piece.row_begin, np.diff(rp_local))
                    cols = piece.col_ind.numpy()
                    ew = (dis_pad[rows] * dis_pad[cols]).astype(np.float32)
                    out[c * mc:c * mc + piece.num_rows] = torch.from_numpy(
                        O.spmm(rp_local, cols, x_pad, mode=O.W_EDGE, ew=ew))
                works.append(dist.all_gather_into_tensor(gathered[c * world * mc:(c + 1) * world * mc],
                                                         out[c * mc:(c + 1) * mc], async_op=True))
            for w in works:
                w.wait()
            results.append(lay.unpad_rows(gathered).numpy())
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_two_rank_padded_allgather_matches_single_rank():
    from oracle import oracle as O
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_padded, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n, f = 1500, 8
    u, v = synth.rmat_undirected(n, 11000, seed=7)
    s, d = synth.symmetrize(u, v)
    g = G.build_gcn_normalized_csr(s, d, num_nodes=n)
    x = synth.features(n, f, seed=8)
    ref = O.spmm(g.row_ptr.numpy(), g.col_ind.numpy(), x.numpy(), mode=O.W_GCN, dis=g.deg_inv_sqrt.numpy())
    for r in range(2):
        for got in results[r]:
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_two_rank_exchange_matches_single_rank():
    from oracle import oracle as O
    from gnn_cuda_b200.GNN_cuda_common import graph_utils as G
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n, f = 1200, 16
    u, v = synth.rmat_undirected(n, 9000, seed=5)
    s, d = synth.symmetrize(u, v)
    g = G.build_gcn_normalized_csr(s, d, num_nodes=n)
    x = synth.features(n, f, seed=6)
    ref = O.spmm(g.row_ptr.numpy(), g.col_ind.numpy(), x.numpy(), mode=O.W_GCN, dis=g.deg_inv_sqrt.numpy())
    for r in range(2):
        assert np.array_equal(results[r].view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("world,chunks,balanced,rank_major", [(2, 1, True, False), (3, 2, True, False),
                                                              (4, 3, False, False), (8, 2, True, False),
                                                              (3, 2, True, True), (8, 2, True, True)])
def test_halo_plan_delivers_every_row_a_rank_reads(world, chunks, balanced, rank_major):
    """Emulates the halo exchange on the CPU: every rank writes its own rows into
    its copy of the next layer's input (the rest NaN), then each rank's listed
    rows are copied into the listed peers' copies. Every row a rank's CSR reads
    must then hold the true value — and nothing beyond the halo is sent."""
    n = 3000
    u, v = synth.rmat_undirected(n, n * 6, seed=71)
    s, d = synth.symmetrize(u, v)
    rp, ci, _ = synth.csr_on_device(s, d, n, add_self_loops=True)
    lay = partition.make_padded_layout(rp.numpy(), world, chunks, balanced=balanced, row_cost=6,
                                       rank_major=rank_major)
    truth = lay.pad_rows(torch.arange(n, dtype=torch.float32).unsqueeze(1) + 1.0)
    ids_of = lay.ids
    bufs = []
    for r in range(world):
        b = torch.full((lay.padded_rows, 1), float("nan"))
        own = ids_of[lay.order[r]]
        b[own] = truth[own]
        bufs.append(b)
    plans = [partition.make_halo_plan(rp, ci, lay, r) for r in range(world)]
    for r, plan in enumerate(plans):
        assert plan.peers == [p for p in range(world) if p != r]
        for c in range(lay.chunks):
            off = plan.offsets[c]
            assert len(off) == world and off[0] == 0
            ids = plan.ids[c].to(torch.int64)
            lo, hi = lay.piece_first(r, c), lay.piece_first(r, c) + lay.chunk_rows
            assert bool(((ids >= lo) & (ids < hi)).all()), "listed rows must be the sender's piece c"
            for q, p in enumerate(plan.peers):
                seg = ids[off[q]:off[q + 1]]
                assert bool((seg[1:] > seg[:-1]).all()), "sorted, no duplicates"
                bufs[p][seg] = bufs[r][seg]
    sent = 0
    for r in range(world):
        shard = partition.make_padded_shard(rp, ci, lay, r)
        cols = torch.cat([pc.col_ind.to(torch.int64) for pc in shard.pieces])
        assert torch.equal(bufs[r][cols], truth[cols]), f"rank {r} reads a row that was not delivered"
        own = set(ids_of[lay.order[r]].tolist())
        sent += len(set(cols.tolist()) - own)
    assert sent == sum(p.rows_sent for p in plans)


@pytest.mark.parametrize("world,chunks,rank_major", [(2, 1, True), (4, 3, True), (8, 2, False), (8, 1, True)])
def test_halo_piece_masks_hold_the_halo_lists(world, chunks, rank_major):
    """Bit q of row i of piece c's mask is set exactly when peers[q]'s list holds that row:
    the form the transform's fused push reads."""
    n = 2500
    u, v = synth.rmat_undirected(n, n * 5, seed=world * 10 + chunks)
    s, d = synth.symmetrize(u, v)
    rp, ci, _ = synth.csr_on_device(s, d, n, add_self_loops=True)
    lay = partition.make_padded_layout(rp.numpy(), world, chunks, balanced=True, row_cost=6, rank_major=rank_major)
    for r in range(world):
        plan = partition.make_halo_plan(rp, ci, lay, r)
        shard = partition.make_padded_shard(rp, ci, lay, r)
        masks = plan.piece_masks(shard)
        assert len(masks) == len(shard.pieces)
        for c, (piece, m) in enumerate(zip(shard.pieces, masks)):
            assert m.dtype == torch.uint8 and m.numel() == piece.num_rows
            want = torch.zeros(piece.num_rows, dtype=torch.int64)
            off = plan.offsets[c]
            for q in range(len(plan.peers)):
                rows = plan.ids[c][off[q]:off[q + 1]].to(torch.int64) - piece.row_begin
                assert bool(((rows >= 0) & (rows < piece.num_rows)).all())
                want[rows] |= 1 << q
            assert torch.equal(m.to(torch.int64), want)
        assert sum(int(torch.bitwise_and(mk.to(torch.int64)[:, None], 1 << torch.arange(8)).ne(0).sum())
                   for mk in masks) == plan.rows_sent
