"""Memory placement policy with the reference's API (GNN_cuda_common/allocator.py:12-191).

``device`` tensors come from PyTorch's caching allocator, ``uvm`` tensors from
cudaMallocManaged through libgnnb200.so, and ``hmm`` tensors are ordinary
pageable CPU tensors read by the GPU through HMM. The mode names, aliases,
error messages and hint semantics are the reference's. Additions: every
prefetch can be issued on a caller-chosen stream (the reference always used the
device's default stream), and ``prefetch_rows_in_order`` issues a row-range
prefetch in row-partition order on a side stream so migration overlaps the
aggregation that consumes the rows.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable

import torch

from .loader import load_allocator_module

DTYPE_TO_CODE = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.int32: 3, torch.int64: 4}
LOCATION_TO_CODE = {"cpu": -1, "cuda": 0}
GRAPH_MEMORY_MODES = ("device", "uvm", "hmm")
COMPUTE_MEMORY_MODES = ("device", "uvm")
WEIGHT_MEMORY_MODES = COMPUTE_MEMORY_MODES
MEMORY_MODE_ALIASES = {"device": "device", "torch_cuda": "device", "uvm": "uvm", "managed": "uvm", "hmm": "hmm"}


@dataclass
class ManagedAllocationConfig:
    preferred_location: str = "cuda"
    accessed_by_cpu: bool = True
    accessed_by_cuda: bool = True
    read_mostly_graph: bool = True
    prefetch_to: str = "cuda"


def normalize_memory_mode(memory_mode: str, *, allow_hmm: bool) -> str:
    normalized = MEMORY_MODE_ALIASES.get(str(memory_mode))
    if normalized is None:
        supported = GRAPH_MEMORY_MODES if allow_hmm else COMPUTE_MEMORY_MODES
        raise ValueError(f"Unsupported memory_mode: {memory_mode}. Expected one of {supported}.")
    if normalized == "hmm" and not allow_hmm:
        raise ValueError("compute memory only supports 'device' or 'uvm'; 'hmm' is graph-only")
    return normalized


def is_uvm_mode(memory_mode: str) -> bool:
    return normalize_memory_mode(memory_mode, allow_hmm=True) == "uvm"


def is_hmm_mode(memory_mode: str) -> bool:
    return normalize_memory_mode(memory_mode, allow_hmm=True) == "hmm"


def uses_cuda_memory_hints(memory_mode: str) -> bool:
    return normalize_memory_mode(memory_mode, allow_hmm=True) in ("uvm", "hmm")


def prefers_hmm_spmm(*memory_modes: str) -> bool:
    return any(normalize_memory_mode(m, allow_hmm=True) == "hmm" for m in memory_modes)


def _device_index(device: torch.device) -> int:
    return int(device.index or 0)


def _dtype_code(dtype: torch.dtype, what: str) -> int:
    code = DTYPE_TO_CODE.get(dtype)
    if code is None:
        raise ValueError(f"Unsupported dtype for {what} allocation: {dtype}")
    return code


def managed_empty(shape: Iterable[int], *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if device.type != "cuda":
        raise ValueError("managed_empty requires a CUDA device")
    return load_allocator_module().managed_empty(list(shape), _dtype_code(dtype, "managed"), _device_index(device))


def hmm_empty(shape: Iterable[int], *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if device.type != "cuda":
        raise ValueError("hmm_empty requires a CUDA device")
    return load_allocator_module().hmm_empty(list(shape), _dtype_code(dtype, "hmm"), _device_index(device))


def allocate_like_mode(cpu_tensor: torch.Tensor, *, memory_mode: str, device: torch.device,
                       uvm_initial_location: str = "cuda") -> torch.Tensor:
    memory_mode = normalize_memory_mode(memory_mode, allow_hmm=True)
    if memory_mode == "uvm":
        out = managed_empty(cpu_tensor.shape, dtype=cpu_tensor.dtype, device=device)
        if uvm_initial_location == "cpu":
            load_allocator_module().copy_cpu_to_managed_(out, cpu_tensor.contiguous())
        elif uvm_initial_location in ("cuda", "none"):
            out.copy_(cpu_tensor, non_blocking=False)
        else:
            raise ValueError("uvm_initial_location expects 'cpu', 'cuda', or 'none'")
        return out
    if memory_mode == "hmm":
        out = hmm_empty(cpu_tensor.shape, dtype=cpu_tensor.dtype, device=device)
        out.copy_(cpu_tensor, non_blocking=False)
        return out
    return cpu_tensor.to(device=device)


def allocate_empty(shape: Iterable[int], *, dtype: torch.dtype, device: torch.device, memory_mode: str) -> torch.Tensor:
    memory_mode = normalize_memory_mode(memory_mode, allow_hmm=True)
    if memory_mode == "uvm":
        return managed_empty(shape, dtype=dtype, device=device)
    if memory_mode == "hmm":
        return hmm_empty(shape, dtype=dtype, device=device)
    return torch.empty(tuple(shape), dtype=dtype, device=device)


def apply_managed_policy(tensor: torch.Tensor, *, device: torch.device, preferred_location: str,
                         accessed_by_cpu: bool, accessed_by_cuda: bool, read_mostly: bool) -> None:
    mod = load_allocator_module()
    idx = _device_index(device)
    if preferred_location != "none":
        mod.advise_preferred_location_(tensor, LOCATION_TO_CODE[preferred_location], idx)
    if accessed_by_cpu:
        mod.advise_accessed_by_(tensor, LOCATION_TO_CODE["cpu"], idx)
    if accessed_by_cuda:
        mod.advise_accessed_by_(tensor, LOCATION_TO_CODE["cuda"], idx)
    if read_mostly:
        mod.advise_read_mostly_(tensor, True)


def prefetch_managed(tensor: torch.Tensor, *, location: str, device: torch.device, nbytes: int | None = None,
                     stream: torch.cuda.Stream | None = None) -> None:
    """Whole-tensor prefetch, or the first ``nbytes`` bytes (allocator.py:170-187)."""
    if location == "none":
        return
    mod = load_allocator_module()
    target = LOCATION_TO_CODE[location]
    if target == 0:
        target = _device_index(device)
    handle = None if stream is None else stream.cuda_stream
    total = int(tensor.numel() * tensor.element_size())
    if nbytes is None:
        mod.prefetch_(tensor, target, _device_index(device), handle)
        return
    byte_count = max(0, min(int(nbytes), total))
    mod.prefetch_range_(tensor, 0, byte_count, target, _device_index(device), handle)


def prefetch_rows_in_order(tensor: torch.Tensor, *, device: torch.device, row_bounds: list[tuple[int, int]],
                           stream: torch.cuda.Stream) -> list[torch.cuda.Event]:
    """Prefetch row ranges of a row-major managed tensor to ``device`` one after
    another on ``stream``; returns one event per range, recorded after its
    prefetch, so a consumer can wait for exactly the rows it reads next."""
    mod = load_allocator_module()
    row_bytes = int(tensor[0].numel() * tensor.element_size()) if tensor.dim() > 1 else int(tensor.element_size())
    events = []
    for r0, r1 in row_bounds:
        mod.prefetch_range_(tensor, int(r0) * row_bytes, int(r1 - r0) * row_bytes, _device_index(device),
                            _device_index(device), stream.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        events.append(ev)
    return events


def pointer_info(tensor: torch.Tensor) -> dict[str, object]:
    return dict(load_allocator_module().pointer_info(tensor))
