"""Row-partitioned multi-GPU GCN forward equals the single-GPU forward bit for bit.

Covers the exchanges: NCCL broadcast; NCCL all_gather on the padded
chunk-major layout; pushes into the peers' IPC-mapped buffers by the SM push
kernel and by copy engines, and halo pushes of only the rows each peer reads
(three steps in a row, so both alternating buffers are used, and the rows a
halo push skips hold stale values that must never be read) — on contiguous
row ranges and on rows dealt to ranks by cost, with 1 to 3 pieces per rank, in
the chunk-major and the rank-major padded layouts (the latter with the last
layer as one call over all of a rank's rows).

Runs on 2 and on 4 GPUs where that many are visible (spawned ranks, one GPU each,
NCCL with NVLS off). The long-row threshold is fixed so every rank uses the
same per-row schedule as the single-GPU run.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
N_NODES, FEAT, LAYERS, THR = 20000, 128, 2, 64


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(device):
    from gnn_cuda_b200 import synth
    u, v = synth.rmat_undirected(N_NODES, N_NODES * 12, seed=61)
    s, d = synth.symmetrize(u, v)
    rp, ci, dis = synth.csr_on_device(s.to(device), d.to(device), N_NODES, add_self_loops=True)
    x = synth.features(N_NODES, FEAT, seed=62).to(device)
    ws = [synth.glorot(FEAT, FEAT, seed=63 + i).to(device) for i in range(LAYERS)]
    bs = [torch.full((FEAT,), 0.01 * (i + 1), device=device) for i in range(LAYERS)]
    return rp, ci, dis, x, ws, bs


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from gnn_cuda_b200 import _native as N
    from gnn_cuda_b200 import partition
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        N.config_set("spmm.long_row_threshold", THR)
        torch.backends.cuda.matmul.allow_tf32 = True
        rp, ci, dis, x, ws, bs = _problem(dev)
        # broadcast exchange over unpadded row ranges
        bounds = partition.nnz_balanced_bounds(rp.cpu().numpy(), world)
        shard = partition.make_shard(rp, ci, bounds[rank], bounds[rank + 1])
        rows = shard.num_rows
        bufs = {k: torch.empty(rows, FEAT, device=dev) for k in ("agg", "out0", "out1")}
        bufs["x_next"] = torch.empty(N_NODES, FEAT, device=dev)
        out = partition.gcn_forward_partitioned(shard, dis, x, ws, bs, bounds, rank, bufs)
        full = torch.empty(N_NODES, FEAT, device=dev)
        partition.exchange_rows(out, full, bounds, rank)
        # padded chunk-major layouts (contiguous ranges or rows dealt by cost), both exchanges
        padded = []
        rp_np = rp.cpu().numpy()
        # (exchange, transport, pieces, rows dealt by cost, rank-major layout); rank-major
        # layouts run the last layer as one call over all of a rank's rows
        cases = [("allgather", None, 1, False, False), ("allgather", None, 3, True, False),
                 ("push", "sm", 1, True, False), ("push", "ce", 3, True, False), ("push", "sm", 2, False, False),
                 ("halo", "sm", 1, True, False), ("halo", "sm", 2, True, False), ("halo", "sm", 3, False, False),
                 ("halo", "sm", 2, True, True), ("push", "sm", 3, False, True), ("halo-graph", "sm", 2, True, True),
                 ("halo-fused", "sm", 1, True, True), ("halo-fused", "sm", 2, False, True),
                 ("halo-fused-graph", "sm", 1, True, True)]
        for how, transport, chunks, balanced, rank_major in cases:
            lay = partition.make_padded_layout(rp_np, world, chunks, balanced=balanced, row_cost=6,
                                               rank_major=rank_major)
            pshard = partition.make_padded_shard(rp, ci, lay, rank)
            dis_p, x_p = lay.pad_rows(dis), lay.pad_rows(x)
            if how == "allgather":
                pbufs = partition.allgather_buffers(lay, FEAT, dev)
                pout = partition.gcn_forward_allgather(pshard, dis_p, x_p, ws, bs, lay, pbufs)
            else:
                ex = partition.PeerRowExchange(lay.padded_rows, FEAT, rank, world, dev, transport=transport)
                halo = partition.make_halo_plan(rp, ci, lay, rank) if how.startswith("halo") else None
                agg = torch.empty(lay.local_rows if rank_major else lay.chunk_rows, FEAT, device=dev)
                mine = torch.empty(lay.local_rows, FEAT, device=dev)

                masks = None
                if "fused" in how:  # the transform stores the halo rows to the peers itself
                    assert N.lib().gnn_gemm_uses_tensor_cores(pshard.pieces[0].num_rows, FEAT, FEAT) == 1
                    masks = halo.piece_masks(pshard)

                def fwd():
                    return partition.gcn_forward_push(pshard, dis_p, x_p, ws, bs, lay, ex, agg, mine, halo=halo,
                                                      push_masks=masks)
                for _ in range(3):  # repeated steps alternate the two copies
                    pout = fwd()
                if how.endswith("graph"):
                    # captured steps replayed in turn, with an eager step between replays
                    mine.fill_(float("nan"))
                    graphs = partition.PushForwardGraphs(fwd, ex)
                    for k in range(5):
                        pout = graphs.replay() if k != 2 else fwd()
                    torch.cuda.synchronize(dev)
                    graphs.close()
            # collect the final rows through the same layout
            pfull = torch.zeros(lay.local_rows, FEAT, device=dev)
            pfull[:pshard.num_rows] = pout
            gathered = torch.empty(lay.padded_rows, FEAT, device=dev)
            mc = lay.chunk_rows
            if rank_major:
                dist.all_gather_into_tensor(gathered, pfull)
            else:
                for c in range(lay.chunks):
                    dist.all_gather_into_tensor(gathered[c * world * mc:(c + 1) * world * mc],
                                                pfull[c * mc:(c + 1) * mc])
            padded.append(lay.unpad_rows(gathered).cpu().numpy())
            if how != "allgather":
                ex.close()
        torch.cuda.synchronize(dev)
        q.put((rank, full.cpu().numpy(), padded))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_partitioned_gcn_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from gnn_cuda_b200 import _native as N
    from gnn_cuda_b200.GNN_cuda_common import agg_ops, gcn_ops
    dev = torch.device("cuda", 0)
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", THR)
    try:
        torch.backends.cuda.matmul.allow_tf32 = True
        rp, ci, dis, x, ws, bs = _problem(dev)
        agg = torch.empty(N_NODES, FEAT, device=dev)
        h = x
        for li in range(LAYERS):
            gcn_ops.spmm_gcn_forward_(rp, ci, dis, h, agg)
            o = torch.empty(N_NODES, FEAT, device=dev)
            agg_ops.linear_forward_(agg, ws[li], bs[li], o, li != LAYERS - 1)
            h = o
        single = h.cpu().numpy()
    finally:
        N.config_set("spmm.long_row_threshold", old)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, bcast, padded = q.get(timeout=300)
        results[r] = (bcast, padded)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert np.array_equal(results[r][0].view(np.uint32), single.view(np.uint32)), ("broadcast", r)
        for k, got in enumerate(results[r][1]):
            assert np.array_equal(got.view(np.uint32), single.view(np.uint32)), ("allgather", k, r)
