#!/usr/bin/env python3
"""Generate the CSR golden vectors by running the reference's own builders.

Imports ``GNN_cuda_common/graph_utils.py`` from the reference checkout (read
only, in the development container; GPU test runs never run this) and records,
for a set of small edge lists that cover the edge cases of the CSR contract
(duplicate edges, pre-existing self-loops, isolated nodes, a single node, an
empty edge list, a power-law graph), the outputs of
  build_gcn_normalized_csr     (graph_utils.py:449-473)
  build_pyg_gcn_weighted_csr   (graph_utils.py:476-504)
  build_plain_csr              (graph_utils.py:507-535, both orientations)
into ``tests/golden/csr_cases.npz``. The tests check both the oracle's
restatement and this package's builders against these arrays bit for bit.

Usage:  python tests/golden/make_golden.py [--reference DIR]  (default: $GNN_REFERENCE_ROOT, else ../reference)
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "csr_cases.npz"


def _load_reference_graph_utils(reference: Path):
    path = reference / "GNN_cuda_common" / "graph_utils.py"
    spec = importlib.util.spec_from_file_location("reference_graph_utils", str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve their module through sys.modules
    spec.loader.exec_module(mod)
    return mod


def _cases() -> dict[str, tuple[np.ndarray, np.ndarray, int]]:
    rng = np.random.default_rng(20261201)
    cases: dict[str, tuple[np.ndarray, np.ndarray, int]] = {}
    # hand-written: duplicates (0->1 twice, 2->1 three times), a self-loop already present (3->3),
    # an isolated node (5), unsorted input order
    src = np.array([0, 2, 0, 2, 3, 4, 2, 1, 4, 0], dtype=np.int64)
    dst = np.array([1, 1, 1, 1, 3, 0, 1, 4, 2, 4], dtype=np.int64)
    cases["handmade"] = (src, dst, 6)
    cases["single_node"] = (np.zeros(0, np.int64), np.zeros(0, np.int64), 1)
    cases["single_node_selfloop"] = (np.zeros(1, np.int64), np.zeros(1, np.int64), 1)
    cases["empty_edges"] = (np.zeros(0, np.int64), np.zeros(0, np.int64), 7)
    # power-law (Chung-Lu style) with duplicates left in
    n = 300
    w = (np.arange(1, n + 1, dtype=np.float64)) ** (-1.0 / 1.1)
    p = w / w.sum()
    m = 2500
    s = rng.choice(n, size=m, p=p)
    d = rng.choice(n, size=m, p=p)
    cases["powerlaw_dups"] = (s.astype(np.int64), d.astype(np.int64), n)
    # a hub row of degree > 1000 (exercises long rows downstream)
    n2 = 1500
    s2 = np.concatenate([np.arange(1, n2), rng.integers(0, n2, 3000)])
    d2 = np.concatenate([np.zeros(n2 - 1, np.int64), rng.integers(0, n2, 3000)])
    cases["hub"] = (s2.astype(np.int64), d2.astype(np.int64), n2)
    return cases


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GNN_REFERENCE_ROOT",
                    str(Path(__file__).resolve().parents[3] / "reference")))
    args = ap.parse_args()
    gu = _load_reference_graph_utils(Path(args.reference))
    arrays: dict[str, np.ndarray] = {}
    for name, (src, dst, n) in _cases().items():
        s_t, d_t = torch.from_numpy(src), torch.from_numpy(dst)
        arrays[f"{name}/src"] = src
        arrays[f"{name}/dst"] = dst
        arrays[f"{name}/num_nodes"] = np.array([n], dtype=np.int64)
        g = gu.build_gcn_normalized_csr(s_t, d_t, num_nodes=n, add_self_loops=True)
        arrays[f"{name}/gcn/row_ptr"] = g.row_ptr.numpy()
        arrays[f"{name}/gcn/col_ind"] = g.col_ind.numpy()
        arrays[f"{name}/gcn/deg_inv_sqrt"] = g.deg_inv_sqrt.numpy()
        g = gu.build_gcn_normalized_csr(s_t, d_t, num_nodes=n, add_self_loops=False)
        arrays[f"{name}/gcn_noloops/row_ptr"] = g.row_ptr.numpy()
        arrays[f"{name}/gcn_noloops/col_ind"] = g.col_ind.numpy()
        arrays[f"{name}/gcn_noloops/deg_inv_sqrt"] = g.deg_inv_sqrt.numpy()
        w = gu.build_pyg_gcn_weighted_csr(s_t, d_t, num_nodes=n, add_self_loops=True)
        arrays[f"{name}/pyg/row_ptr"] = w.row_ptr.numpy()
        arrays[f"{name}/pyg/col_ind"] = w.col_ind.numpy()
        arrays[f"{name}/pyg/edge_weight"] = w.edge_weight.numpy()
        for loops in (False, True):
            for tr in (True, False):
                p = gu.build_plain_csr(s_t, d_t, num_nodes=n, add_self_loops=loops, transpose_for_incoming=tr)
                key = f"{name}/plain_l{int(loops)}_t{int(tr)}"
                arrays[f"{key}/row_ptr"] = p.row_ptr.numpy()
                arrays[f"{key}/col_ind"] = p.col_ind.numpy()
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays)} arrays)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
