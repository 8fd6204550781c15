"""The locality-preprocessing oracle against the reference's own outputs.

``tests/golden/locality_cases.npz`` holds what the reference's
build_page_reuse_schedule_metadata / build_coaccess_feature_permutation /
build_hot_partition_feature_permutation (graph_utils.py:174-446) returned,
chained as run/preprocess_gcn_graph.py:40-120 chains them. The oracle must
reproduce every array and scalar bit for bit before the device implementation
is checked against it.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import locality as L

GOLDEN = Path(__file__).resolve().parent / "golden" / "locality_cases.npz"

PAGE_ARRAYS = ("page_histogram", "page_reuse_histogram", "hot_pages", "row_schedule", "block_hot_pages",
               "window_hot_pages")
PAGE_SCALARS = ("rows_per_page", "num_pages", "row_block_size", "window_num_blocks", "window_cache_pages",
                "rows_per_window", "signature_topk", "page_bytes", "hot_coverage", "avg_window_hot_coverage")
HOT_ARRAYS = ("perm", "inv_perm", "hot_nodes", "hot_node_access_counts")
HOT_SCALARS = ("hot_node_cutoff", "hot_total_accesses", "hot_min_nodes", "hot_node_fraction",
               "hot_node_access_coverage", "hot_access_target", "hot_max_ratio")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def case_names():
    return [str(c) for c in np.load(GOLDEN)["cases"]]


def params(g, name):
    out = {}
    for k in ("feat_dim", "page_bytes", "row_block_size", "window_num_blocks", "window_cache_pages",
              "hot_cache_pages", "signature_topk", "hot_min_nodes"):
        out[k] = int(g[f"{name}/param/{k}"][0])
    for k in ("hot_access_coverage", "hot_max_ratio"):
        out[k] = float(g[f"{name}/param/{k}"][0])
    return out


def check_page(meta: dict, g, key: str) -> None:
    for k in PAGE_ARRAYS:
        exp = g[f"{key}/{k}"]
        got = np.asarray(meta[k])
        assert got.dtype == np.int64 and got.shape == exp.shape and np.array_equal(got, exp), f"{key}/{k}"
    for k in PAGE_SCALARS:
        exp = g[f"{key}/{k}"][0]
        got = meta[k]
        assert float(got) == float(exp), f"{key}/{k}: {got!r} != {exp!r}"


def check_hot(hot: dict, g, key: str) -> None:
    for k in HOT_ARRAYS:
        exp = g[f"{key}/{k}"]
        got = np.asarray(hot[k])
        assert got.shape == exp.shape and np.array_equal(got, exp), f"{key}/{k}"
    for k in HOT_SCALARS:
        assert float(hot[k]) == float(g[f"{key}/{k}"][0]), f"{key}/{k}"


@pytest.mark.parametrize("name", case_names())
def test_oracle_pipeline_matches_reference(gold, name):
    src, dst = gold[f"{name}/src"], gold[f"{name}/dst"]
    n = int(gold[f"{name}/num_nodes"][0])
    res = L.preprocess(src, dst, num_nodes=n, **params(gold, name))
    check_page(res["base"], gold, f"{name}/base")
    assert np.array_equal(res["coaccess_perm"], gold[f"{name}/coaccess/perm"])
    check_hot(res["hot"], gold, f"{name}/hot")
    if f"{name}/reordered/src" in gold.files:
        assert np.array_equal(res["src"], gold[f"{name}/reordered/src"])
        assert np.array_equal(res["dst"], gold[f"{name}/reordered/dst"])
    check_page(res["final"], gold, f"{name}/final")


@pytest.mark.parametrize("name", case_names())
def test_oracle_hot_partition_without_base(gold, name):
    src = gold[f"{name}/src"]
    n = int(gold[f"{name}/num_nodes"][0])
    p = params(gold, name)
    hot = L.hot_partition(src, num_nodes=n, hot_access_coverage=p["hot_access_coverage"],
                          hot_max_ratio=p["hot_max_ratio"], hot_min_nodes=p["hot_min_nodes"])
    check_hot(hot, gold, f"{name}/hot_nobase")
