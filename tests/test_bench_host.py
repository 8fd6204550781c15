"""Host-side pieces of bench.py that need no GPU: the defaults a plain
`bench.py --gpus N` (the driver's command line) runs with, the pieces-per-rank
rule, the configuration label, and the clock sampler on ranks that do not sample.
"""
import sys

import pytest

import bench


def _args(monkeypatch, *argv):
    monkeypatch.setattr(sys, "argv", ["bench.py", *argv])
    return bench.parse_args()


def test_driver_command_line_defaults(monkeypatch):
    a = _args(monkeypatch, "--gpus", "8", "--steps", "20", "--warmup", "5")
    assert (a.gpus, a.steps, a.warmup, a.impl) == (8, 20, 5, "ours")
    # the multi-GPU path measured best: halo rows stored by the transform's epilogue,
    # rank-major rows, one piece per rank, one long-row threshold per shard, graph replays
    assert a.exchange == "halo" and a.push_from == "transform" and a.padded_order == "rank"
    assert a.layout == "balanced" and a.long_rows == "shard" and a.graphs and a.check
    assert bench.default_chunks(a.chunks, 8) == 1 and bench.default_chunks(3, 8) == 3
    a = _args(monkeypatch)
    assert a.gpus == 1 and a.warmup >= 3 and a.workload == "gcn_products_like"


def test_configuration_label_names_the_exchange():
    prob = {"n": 10, "nnz": 20}
    d = bench.describe(prob, 8, gemm="tcgen05-tf32", chunks=1, order="row id")
    assert d["parallelism"] == "rows8+balanced_halo_push_pieces1_rank_major_from_transform"
    d = bench.describe(prob, 8, gemm="tcgen05-tf32", chunks=2, order="row id", push_from="kernel",
                       padded_order="chunk")
    assert d["parallelism"] == "rows8+balanced_halo_push_pieces2_chunk_major"
    assert bench.describe(prob, 1, gemm="g", order="o")["parallelism"] == "rows1"


@pytest.mark.parametrize("enabled", [False])
def test_a_disabled_clock_sampler_starts_nothing(enabled):
    with bench.ClockSampler(0, enabled=enabled) as c:
        assert c.proc is None
    assert c.summary()["sm_mhz"] is None
