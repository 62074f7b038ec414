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


def stream_handle(device: torch.device) -> ctypes.c_void_p:
    """Raw cudaStream_t of the caller's current stream (what Triton launches on)."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Device scratch of at least ``nbytes`` reserved per (device, stream, size).

    Workspaces are never freed or resized: a CUDA graph that captured a launch keeps
    pointing at the same bytes for as long as the process lives.  Launches on one
    stream are ordered, so they can share the bytes; another stream gets its own.
    """
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream, int(nbytes))
    with _workspace_lock:
        buffer = _workspaces.get(key)
        if buffer is None:
            buffer = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)
            _workspaces[key] = buffer
    return buffer


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()
