"""Module loaders with the reference's names (GNN_cuda_common/loader.py:62-99).

The reference JIT-compiles four PyTorch extensions on first use. Here a single
prebuilt C-ABI library (libgnnb200.so, built by ``gnn_cuda_b200/build.py`` for
sm_100a) backs all four tables; each loader returns a namespace exposing the
same function names as the corresponding pybind11 module. A missing library
raises RuntimeError: there is no fallback implementation.
"""
from __future__ import annotations

from .. import _native
from . import native_ops


def _ensure_loaded():
    _native.lib()


def load_allocator_module():
    _ensure_loaded()
    return native_ops.ALLOCATOR_MODULE


def load_gcn_module():
    _ensure_loaded()
    return native_ops.GCN_MODULE


def load_pyg_gcn_module():
    _ensure_loaded()
    return native_ops.PYG_GCN_MODULE


def load_agg_module():
    _ensure_loaded()
    return native_ops.AGG_MODULE
