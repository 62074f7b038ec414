"""Host plumbing shared by the operator wrappers: dtype codes, streams, workspaces.

PyTorch only supplies device memory and the current CUDA stream here; every kernel
runs from libjetspec_b200.so through the C ABI.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

DTYPE_CODES = {torch.bfloat16: _lib.JT_BF16, torch.float16: _lib.JT_F16,
               torch.float32: _lib.JT_F32}

_workspaces: dict = {}
_workspace_lock = threading.Lock()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def raw_stream(device: torch.device) -> int:
    """cudaStream_t (as an int) of the caller's current stream on ``device``, without
    building a torch Stream object (a few microseconds per call saved on the launch path)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(device).cuda_stream


def stream_handle(device: torch.device) -> ctypes.c_void_p:
    """Raw cudaStream_t of the caller's current stream (what Triton launches on)."""
    return ctypes.c_void_p(raw_stream(device))


def workspace(device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
    """Device scratch of at least ``nbytes`` reserved per (device, stream, size).

    Workspaces are never freed or resized: a CUDA graph that captured a launch keeps
    pointing at the same bytes for as long as the process lives.  Launches on one
    stream are ordered, so they can share the bytes; another stream gets its own.
    """
    if stream is None:
        stream = raw_stream(device)
    key = (device.index, stream, int(nbytes))
    with _workspace_lock:
        buffer = _workspaces.get(key)
        if buffer is None:
            buffer = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)
            _workspaces[key] = buffer
    return buffer


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()
