"""The transform with the halo push in its epilogue (gnn_linear_push_forward), on one GPU.

The destinations are ordinary buffers on the same GPU standing in for the
peers' copies (the kernel stores to whatever device addresses it is given; the
multi-GPU test covers real peer buffers). Every output row must equal the plain
transform's bit for bit, every row whose mask bit d is set must appear in
destination d, and every other destination row must be left untouched.
"""
import numpy as np
import pytest
import torch

from gnn_cuda_b200 import _native as N
from gnn_cuda_b200 import synth
from gnn_cuda_b200.GNN_cuda_common import native_ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _bits(t):
    return t.detach().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("m,k,n,npeers,relu", [(20011, 128, 128, 7, True), (777, 64, 128, 3, False),
                                               (4096, 128, 64, 8, True), (130, 32, 32, 1, True),
                                               (50000, 256, 128, 5, False)])
def test_rows_reach_exactly_the_masked_destinations(m, k, n, npeers, relu):
    g = torch.Generator(device=DEV).manual_seed(m + npeers)
    x = torch.randn(m, k, generator=g, device=DEV)
    w = synth.glorot(k, n, seed=7, device=DEV)
    b = torch.randn(n, generator=g, device=DEV)
    ref = torch.empty(m, n, device=DEV)
    native_ops.linear_forward_(x, w, b, ref, relu)
    # about a third of the rows go nowhere; the rest to a random subset of destinations
    mask = torch.randint(0, 1 << npeers, (m,), generator=g, device=DEV).to(torch.uint8)
    mask[torch.rand(m, generator=g, device=DEV) < 0.33] = 0
    dsts = [torch.full((m, n), float("nan"), device=DEV) for _ in range(npeers)]
    out = torch.full((m, n), float("nan"), device=DEV)
    assert native_ops.linear_push_forward_(x, w, b, out, relu, mask, [d.data_ptr() for d in dsts])
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), _bits(ref))
    mk = mask.cpu().numpy()
    for d, dst in enumerate(dsts):
        sent = (mk >> d) & 1 == 1
        got = dst.cpu().numpy()
        assert np.array_equal(got[sent].view(np.uint32), _bits(ref)[sent]), d
        assert np.isnan(got[~sent]).all(), d


def test_no_destinations_is_the_plain_transform():
    m, k, n = 3000, 128, 128
    x = synth.features(m, k, seed=3, device=DEV)
    w = synth.glorot(k, n, seed=4, device=DEV)
    ref = torch.empty(m, n, device=DEV)
    native_ops.linear_forward_(x, w, None, ref, True)
    out = torch.empty(m, n, device=DEV)
    assert native_ops.linear_push_forward_(x, w, None, out, True, torch.zeros(m, dtype=torch.uint8, device=DEV), [])
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), _bits(ref))


def test_shapes_off_the_tensor_core_path_launch_nothing():
    m, k, n = 100, 48, 128  # K not a multiple of 32: the tensor-core GEMM does not apply
    x = torch.randn(m, k, device=DEV)
    w = torch.randn(k, n, device=DEV)
    out = torch.zeros(m, n, device=DEV)
    dst = torch.zeros(m, n, device=DEV)
    mask = torch.ones(m, dtype=torch.uint8, device=DEV)
    assert not native_ops.linear_push_forward_(x, w, None, out, False, mask, [dst.data_ptr()])
    torch.cuda.synchronize()
    assert not out.any() and not dst.any()
    rc = N.lib().gnn_linear_push_forward(None, None, None, None, 1, 32, 32, 0, None, None, 9, None)
    assert rc != 0 and "npeers" in N.last_error()
