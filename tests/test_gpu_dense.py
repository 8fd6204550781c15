"""GPU parity of the dense transform and the elementwise epilogues (run with -m gpu).

FP32 precision: the FFMA kernel accumulates k in increasing order, exactly
like the oracle's fmaf loop, so results are compared bit for bit. TF32
precision (tensor cores) is held to a 2e-3 relative tolerance,
measured against the float64 product and scaled by sum_k |x_ik * w_kj|.
Elementwise ops are bit-exact with the reference arithmetic.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from gnn_cuda_b200 import _native as N
from gnn_cuda_b200.GNN_cuda_common import agg_ops, native_ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

SHAPES = [(1, 1, 1), (7, 3, 5), (128, 128, 128), (1000, 128, 128), (333, 256, 256), (515, 129, 77),
          (4096, 512, 512), (300, 64, 200)]


def _rand(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g)


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_gemm_fp32_bit_exact(m, k, n):
    x, w = _rand((m, k), 1), _rand((k, n), 2)
    out = torch.empty(m, n, device=DEV)
    native_ops.gemm_forward_(x.to(DEV), w.to(DEV), out, precision=N.GNN_PRECISION_FP32)
    exp = O.gemm_fp32(x.numpy(), w.numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("relu", [False, True])
def test_linear_tf32_within_tolerance(m, k, n, relu):
    x, w, b = _rand((m, k), 3), _rand((k, n), 4), _rand((n,), 5)
    out = torch.empty(m, n, device=DEV)
    native_ops.linear_forward_(x.to(DEV), w.to(DEV), b.to(DEV), out, relu, precision=N.GNN_PRECISION_TF32)
    ref = O.gemm_f64(x.numpy(), w.numpy(), b.numpy(), relu)
    scale = np.abs(x.numpy()).astype(np.float64) @ np.abs(w.numpy()).astype(np.float64) + np.abs(b.numpy())[None, :]
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= 2e-3 * scale + 1e-30), float(np.max(err / (scale + 1e-30)))


TC_SHAPES = [(100_000, 128, 128), (70_000, 256, 256), (5000, 128, 64), (5000, 64, 32), (257, 32, 128),
             (130, 128, 256), (1, 128, 128), (128 * 148 * 3 + 5, 128, 128)]


@pytest.mark.parametrize("m,k,n", TC_SHAPES)
def test_tensor_core_gemm_shapes(m, k, n):
    """Shapes routed to the tcgen05 kernel: TF32 tolerance, and no bounded wait gave up."""
    assert N.lib().gnn_gemm_uses_tensor_cores(m, k, n) == 1
    x, w, b = _rand((m, k), 21), _rand((k, n), 22), _rand((n,), 23)
    out = torch.full((m, n), float("nan"), device=DEV)
    native_ops.linear_forward_(x.to(DEV), w.to(DEV), b.to(DEV), out, True, precision=N.GNN_PRECISION_TF32)
    import ctypes
    status = ctypes.c_int(-1)
    N.check(N.lib().gnn_device_status(1, ctypes.byref(status)))
    assert status.value == 0
    got = out.cpu().numpy().astype(np.float64)
    ref = x.numpy().astype(np.float64) @ w.numpy().astype(np.float64) + b.numpy()[None, :]
    ref = np.maximum(ref, 0.0)
    scale = np.abs(x.numpy()).astype(np.float64) @ np.abs(w.numpy()).astype(np.float64) + np.abs(b.numpy())[None, :]
    assert np.all(np.abs(got - ref) <= 2e-3 * scale + 1e-30)
    # and it really is TF32, not FP32: the error is above FP32 rounding somewhere
    assert np.max(np.abs(got - ref) / (scale + 1e-30)) > 1e-6


def test_linear_fp32_bit_exact_with_bias_relu():
    x, w, b = _rand((777, 128), 6), _rand((128, 96), 7), _rand((96,), 8)
    out = torch.empty(777, 96, device=DEV)
    native_ops.linear_forward_(x.to(DEV), w.to(DEV), b.to(DEV), out, True, precision=N.GNN_PRECISION_FP32)
    exp = O.gemm_fp32(x.numpy(), w.numpy(), b.numpy(), True)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))


def test_gemm_precision_follows_torch_tf32_flag():
    old = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        assert native_ops.gemm_precision() == N.GNN_PRECISION_FP32
        torch.backends.cuda.matmul.allow_tf32 = True
        assert native_ops.gemm_precision() == N.GNN_PRECISION_TF32
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("rows,cols", [(10, 7), (64, 128), (3, 4)])
@pytest.mark.parametrize("relu", [False, True])
def test_bias_relu_bit_exact(rows, cols, relu):
    a, b = _rand((rows, cols), 9), _rand((cols,), 10)
    t = a.to(DEV)
    agg_ops.bias_relu_forward_(t, b.to(DEV), relu)
    exp = O.bias_relu(a.numpy(), b.numpy(), relu)
    assert np.array_equal(t.cpu().numpy().view(np.uint32), exp.view(np.uint32))
    # empty bias: relu only (or a no-op)
    t2 = a.to(DEV)
    agg_ops.bias_relu_forward_(t2, torch.empty(0, device=DEV), relu)
    assert np.array_equal(t2.cpu().numpy().view(np.uint32), O.bias_relu(a.numpy(), None, relu).view(np.uint32))


@pytest.mark.parametrize("count", [1, 5, 4096, 100003])
def test_add_and_relu_inplace_bit_exact(count):
    a, b = _rand((count,), 11), _rand((count,), 12)
    t = a.to(DEV)
    agg_ops.tensor_add_inplace_(t, b.to(DEV), 1.37)
    exp = O.add_inplace(a.numpy(), b.numpy(), np.float32(1.37))
    assert np.array_equal(t.cpu().numpy().view(np.uint32), exp.view(np.uint32))
    agg_ops.relu_inplace_(t)
    assert np.array_equal(t.cpu().numpy().view(np.uint32), O.relu(exp).view(np.uint32))


def test_add_inplace_unaligned_tail():
    a, b = _rand((1001,), 13), _rand((1001,), 14)
    ta, tb = a.to(DEV), b.to(DEV)
    agg_ops.tensor_add_inplace_(ta[1:], tb[1:], 0.5)
    exp = a.numpy().copy()
    exp[1:] = O.add_inplace(a.numpy()[1:], b.numpy()[1:], np.float32(0.5))
    assert np.array_equal(ta.cpu().numpy().view(np.uint32), exp.view(np.uint32))
