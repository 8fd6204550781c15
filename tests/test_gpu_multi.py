"""Row-partitioned multi-GPU GCN forward equals the single-GPU forward bit for bit.

Covers the three exchanges: NCCL broadcast, NCCL all_gather on the padded
chunk-major layout (1 and 3 pieces), and copy-engine pushes into the peers'
IPC-mapped buffers (1 and 3 pieces, three steps in a row so both of the
alternating buffers are used).

Runs only where at least two GPUs are visible (spawned ranks, one GPU each,
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
        # padded chunk-major layout, pipelined all_gather per row piece
        padded = []
        for chunks in (1, 3):
            lay = partition.make_padded_layout(rp.cpu().numpy(), world, chunks)
            pshard = partition.make_padded_shard(rp, ci, lay, rank)
            pbufs = partition.allgather_buffers(lay, FEAT, dev)
            pout = partition.gcn_forward_allgather(pshard, lay.pad_rows(dis), lay.pad_rows(x), ws, bs, lay, pbufs)
            # collect the final rows through the same layout
            pfull = torch.zeros(lay.local_rows, FEAT, device=dev)
            pfull[:pshard.num_rows] = pout
            gathered = torch.empty(lay.padded_rows, FEAT, device=dev)
            for c in range(lay.chunks):
                mc = lay.chunk_rows
                dist.all_gather_into_tensor(gathered[c * world * mc:(c + 1) * world * mc], pfull[c * mc:(c + 1) * mc])
            padded.append(lay.unpad_rows(gathered).cpu().numpy())
        # copy-engine pushes over IPC mappings, pieces of equal nnz
        for chunks in (1, 3):
            pieces = partition.make_pieces(rp, ci, bounds[rank], bounds[rank + 1], chunks)
            ex = partition.PeerRowExchange(N_NODES, FEAT, rank, world, dev)
            agg = torch.empty(max(p.num_rows for p in pieces), FEAT, device=dev)
            mine = torch.empty(rows, FEAT, device=dev)
            for _ in range(3):  # repeated steps alternate the two copies
                partition.gcn_forward_push(pieces, dis, x, ws, bs, ex, agg, mine)
            full_p = torch.empty(N_NODES, FEAT, device=dev)
            partition.exchange_rows(mine, full_p, bounds, rank)
            torch.cuda.synchronize(dev)
            padded.append(full_p.cpu().numpy())
            ex.close()
        torch.cuda.synchronize(dev)
        q.put((rank, full.cpu().numpy(), padded))
    finally:
        dist.destroy_process_group()


def test_two_gpu_partitioned_gcn_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
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
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        r, bcast, padded = q.get(timeout=300)
        results[r] = (bcast, padded)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        assert np.array_equal(results[r][0].view(np.uint32), single.view(np.uint32)), ("broadcast", r)
        for k, got in enumerate(results[r][1]):
            assert np.array_equal(got.view(np.uint32), single.view(np.uint32)), ("allgather", k, r)
