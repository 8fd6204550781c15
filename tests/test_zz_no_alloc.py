"""The allocation-free GCN aggregation entry point (gnn_spmm_gcn_forward_noalloc).

It serves callers that cannot give the library a scratch buffer or let it
allocate device memory (a plugin host that owns all device memory, a process
at a fixed memory budget, a path that must not wait on cudaMalloc/cudaFree).
It must return exactly what gnn_spmm_gcn_forward returns with a caller
workspace — checked on two calls in a row, on a graph whose hub rows make the
kernels use the scratch (the long-row list and its counters), so a second call
that saw stale counters would differ. Sizes past the built-in 8 MiB scratch
must be refused before any work is queued.

The file name sorts last so that a run stopping at the first failure has run
every other test first; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from gnn_cuda_b200 import _native as N
from gnn_cuda_b200 import synth

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _hub_graph(n: int, f: int = 128):
    g = torch.Generator().manual_seed(77)
    # node 0 is a hub of degree n-1; the rest is a sparse random graph
    m = max(20000, 4 * n)
    u = torch.cat([torch.zeros(n - 1, dtype=torch.int64), torch.randint(1, n, (m,), generator=g)])
    v = torch.cat([torch.arange(1, n, dtype=torch.int64), torch.randint(1, n, (m,), generator=g)])
    keep = u != v
    key = torch.unique(torch.minimum(u[keep], v[keep]) * n + torch.maximum(u[keep], v[keep]))
    s, d = synth.symmetrize(key // n, key % n)
    rp, ci, dis = synth.csr_on_device(s, d, n, add_self_loops=True)
    x = synth.features(n, f, seed=78)
    return {k: t.to(DEV).contiguous() for k, t in dict(rp=rp, ci=ci, dis=dis, x=x).items()} | {"n": n, "f": f}


# 6,000 nodes: below the size at which the workspace entry point builds a
# degree-ordered row schedule; 70,000 nodes: above it, where only a workspace
# larger than the minimum would enable that schedule
@pytest.fixture(params=[6000, 70000])
def hub_graph(request):
    return _hub_graph(request.param)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_entry_point_twice(hub_graph):
    g = hub_graph
    n, f, nnz = g["n"], g["f"], g["ci"].numel()
    L = N.lib()
    old = N.config_get("spmm.long_row_threshold")
    N.config_set("spmm.long_row_threshold", 64)  # the hub and many rows go through the scratch list
    try:
        stream = torch.cuda.current_stream(DEV).cuda_stream
        # the minimum workspace, which is what the allocation-free entry point uses
        ws_bytes = L.gnn_spmm_workspace_bytes(n, nnz)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        ref = torch.empty(n, f, device=DEV)
        N.check(L.gnn_spmm_gcn_forward(_ptr(g["rp"]), N.GNN_INDEX_INT32, _ptr(g["ci"]), _ptr(g["dis"]),
                                       _ptr(g["x"]), _ptr(ref), n, nnz, f, _ptr(ws), ws_bytes,
                                       ctypes.c_void_p(stream)))
        outs = []
        for _ in range(2):
            out = torch.full((n, f), float("nan"), device=DEV)
            N.check(L.gnn_spmm_gcn_forward_noalloc(_ptr(g["rp"]), N.GNN_INDEX_INT32, _ptr(g["ci"]), _ptr(g["dis"]),
                                                   _ptr(g["x"]), _ptr(out), n, nnz, f, ctypes.c_void_p(stream)))
            outs.append(out)
        torch.cuda.synchronize(DEV)
        ref_bits = ref.cpu().numpy().view(np.uint32)
        for out in outs:
            # the repository's aggregation tolerance is bit-exactness for a fixed schedule
            assert np.array_equal(out.cpu().numpy().view(np.uint32), ref_bits)
        assert torch.isfinite(ref).all()
    finally:
        N.config_set("spmm.long_row_threshold", old)


def test_noalloc_refuses_problems_beyond_its_scratch():
    L = N.lib()
    # 3,000,000 nodes and 200,000,000 edges need more than 8 MiB of scratch
    rc = L.gnn_spmm_gcn_forward_noalloc(None, N.GNN_INDEX_INT32, None, None, None, None, 3_000_000, 200_000_000,
                                        128, None)
    assert rc == 3  # GNN_ERR_UNSUPPORTED
    msg = N.last_error()
    assert "8388608" in msg and "gnn_spmm_gcn_forward with a workspace" in msg
    # the documented examples fit
    assert L.gnn_spmm_workspace_bytes(1_000_000, 500_000_000) <= 8 << 20
    assert L.gnn_spmm_workspace_bytes(2_449_029, 64_308_169) <= 8 << 20
