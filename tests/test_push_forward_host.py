"""Control flow of partition.gcn_forward_push, without a GPU.

The aggregation and transform calls are replaced by recorders and the exchange
by a fake, so the test sees which calls a step makes: one aggregation and one
transform per piece, pushes only after layers that are followed by another,
one barrier per layer boundary, the last layer as one call over a rank's rows
when they are one block, the transform's fused push when row masks are given,
and the separate push when the fused kernel does not apply.
"""
import pytest
import torch

from gnn_cuda_b200 import partition
from gnn_cuda_b200.GNN_cuda_common import native_ops


class _Exchange:
    transport = "sm"

    def __init__(self, rows: int, feat: int):
        self.turn = 0
        self.copies = [torch.zeros(rows, feat), torch.zeros(rows, feat)]
        self.streams = {}
        self.log = []

    def buffer(self):
        return self.copies[self.turn]

    def push_rows(self, ids, offsets, peers, ready):
        self.log.append(("push", self.turn, int(ids.numel())))

    def push(self, lo, hi, ready):
        self.log.append(("push_range", self.turn, lo, hi))

    def peer_rows(self, row_begin, peers):
        return [1000 * (p + 1) + row_begin for p in peers]

    def finish(self):
        self.log.append(("barrier", self.turn))
        done = self.copies[self.turn]
        self.turn ^= 1
        return done


class _Event:
    def record(self, stream=None):
        pass


@pytest.fixture
def recorder(monkeypatch):
    calls = []
    monkeypatch.setattr(partition, "spmm_gcn_shard",
                        lambda piece, dis, h, a: calls.append(("aggregate", piece.row_begin, piece.num_rows)))
    monkeypatch.setattr(native_ops, "linear_forward_",
                        lambda a, w, b, dst, relu: calls.append(("transform", int(a.size(0)), bool(relu))))
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    return calls


def _setup(world, chunks, rank_major, rank=0, n=1200):
    from gnn_cuda_b200 import synth
    u, v = synth.rmat_undirected(n, n * 5, seed=3)
    s, d = synth.symmetrize(u, v)
    rp, ci, _ = synth.csr_on_device(s, d, n, add_self_loops=True)
    lay = partition.make_padded_layout(rp.numpy(), world, chunks, balanced=True, row_cost=6, rank_major=rank_major)
    shard = partition.make_padded_shard(rp, ci, lay, rank)
    halo = partition.make_halo_plan(rp, ci, lay, rank)
    return lay, shard, halo


def _run(lay, shard, halo, agg_rows, masks=None, layers=3):
    f = 8
    ex = _Exchange(lay.padded_rows, f)
    agg = torch.zeros(agg_rows, f)
    out = torch.zeros(lay.local_rows, f)
    ws = [torch.zeros(f, f)] * layers
    bs = [torch.zeros(f)] * layers
    partition.gcn_forward_push(shard, torch.zeros(lay.padded_rows), torch.zeros(lay.padded_rows, f), ws, bs, lay, ex,
                               agg, out, halo=halo, push_masks=masks)
    return ex


@pytest.mark.parametrize("rank_major", [False, True])
def test_pieces_pushes_and_barriers(recorder, rank_major):
    lay, shard, halo = _setup(4, 3, rank_major)
    ex = _run(lay, shard, halo, agg_rows=lay.local_rows)
    pieces = [p for p in shard.pieces if p.num_rows]
    per_layer = [c for c in recorder if c[0] == "aggregate"]
    # layers 0 and 1 in pieces; the last layer in one call when the rows are one block
    last = 1 if rank_major else len(pieces)
    assert len(per_layer) == 2 * len(pieces) + last
    if rank_major:
        assert per_layer[-1] == ("aggregate", shard.whole.row_begin, shard.num_rows)
    transforms = [c for c in recorder if c[0] == "transform"]
    assert [t[2] for t in transforms] == [True] * (2 * len(pieces)) + [False] * last  # ReLU on all but the last
    # every piece of layers 0 and 1 pushed into the copy of its exchange, then one barrier
    assert ex.log == ([("push", 0, int(halo.ids[c].numel())) for c, p in enumerate(shard.pieces) if p.num_rows] +
                      [("barrier", 0)] +
                      [("push", 1, int(halo.ids[c].numel())) for c, p in enumerate(shard.pieces) if p.num_rows] +
                      [("barrier", 1)])


def test_small_scratch_keeps_the_last_layer_in_pieces(recorder):
    lay, shard, halo = _setup(2, 2, True)
    _run(lay, shard, halo, agg_rows=lay.chunk_rows)
    pieces = [p for p in shard.pieces if p.num_rows]
    assert len([c for c in recorder if c[0] == "aggregate"]) == 3 * len(pieces)


@pytest.mark.parametrize("fused_runs", [True, False])
def test_fused_push_replaces_the_push_kernel(recorder, monkeypatch, fused_runs):
    lay, shard, halo = _setup(4, 1, True)
    masks = halo.piece_masks(shard)
    seen = []

    def fake_push_forward(a, w, b, dst, relu, mask, peer_rows):
        seen.append((int(a.size(0)), relu, mask is masks[0], list(peer_rows)))
        return fused_runs  # False: the tensor-core GEMM does not apply, nothing launched
    monkeypatch.setattr(native_ops, "linear_push_forward_", fake_push_forward)
    ex = _run(lay, shard, halo, agg_rows=lay.local_rows, masks=masks, layers=2)
    # layer 0 only (the last layer pushes nothing); peers addressed at the piece's first row
    assert seen == [(shard.num_rows, True, True, [1000 * (p + 1) + shard.pieces[0].row_begin for p in halo.peers])]
    transforms = [c for c in recorder if c[0] == "transform"]
    if fused_runs:
        assert ex.log == [("barrier", 0)] and transforms == [("transform", shard.num_rows, False)]
    else:
        assert ex.log == [("push", 0, int(halo.ids[0].numel())), ("barrier", 0)]
        assert transforms == [("transform", shard.num_rows, True), ("transform", shard.num_rows, False)]
