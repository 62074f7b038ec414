"""Paged KV store: drop-in for ``store_kvcache`` (nanovllm/layers/attention.py:38-45).

Same signature, same assertions (AssertionError on a layout the reference rejects),
same semantics: ``k_cache[slot] = key[i]`` and ``v_cache[slot] = value[i]`` for every
token whose slot is not -1, bit for bit.
"""
from __future__ import annotations

import ctypes

import torch

from . import _launch, _lib


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    from . import ops

    if ops.compiling():
        torch.ops.jetspec_b200.kv_store_(key, value, k_cache, v_cache, slot_mapping)
        return
    _store(key, value, k_cache, v_cache, slot_mapping)


def _store(key, value, k_cache, v_cache, slots) -> None:
    """Launch jt_kv_store_launch for [N, heads, dim] rows into [blocks, bs, heads, dim]."""
    if int(key.shape[0]) == 0:
        return
    if k_cache.ndim != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("KV caches must be [blocks, block_size, kv_heads, head_dim]")
    if tuple(key.shape) != tuple(value.shape) or tuple(key.shape[1:]) != tuple(k_cache.shape[2:]):
        raise ValueError("key/value rows do not match the cache head geometry")
    if key.dtype != value.dtype or key.dtype != k_cache.dtype or k_cache.dtype != v_cache.dtype:
        raise ValueError("key, value and caches must share one dtype")
    if key.element_size() not in (2, 4):
        raise ValueError("KV store supports 2- or 4-byte elements")
    if slots.dtype not in (torch.int32, torch.int64) or slots.ndim != 1:
        raise ValueError("slot mapping must be a 1-D int32 or int64 tensor")
    tensors = (key, value, k_cache, v_cache, slots)
    if any(not t.is_cuda or t.device != key.device for t in tensors):
        raise ValueError("KV store requires CUDA tensors on one device")
    if (key.stride(-1) != 1 or value.stride(-1) != 1 or k_cache.stride(-1) != 1
            or v_cache.stride(-1) != 1 or not slots.is_contiguous()):
        raise ValueError("KV store needs contiguous head dimensions and slot vector")
    lib = _lib.load_library()
    p = _lib.JtKvStoreParams()
    p.key, p.value = key.data_ptr(), value.data_ptr()
    p.k_cache, p.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    p.slot_mapping = slots.data_ptr()
    p.slot_is_int64 = int(slots.dtype == torch.int64)
    p.num_tokens = int(key.shape[0])
    p.num_kv_heads, p.head_dim = int(key.shape[1]), int(key.shape[2])
    p.elem_bytes = key.element_size()
    p.block_size = int(k_cache.shape[1])
    p.num_blocks = int(k_cache.shape[0])
    p.key_stride0, p.key_stride1 = key.stride(0), key.stride(1)
    p.value_stride0, p.value_stride1 = value.stride(0), value.stride(1)
    p.k_stride0, p.k_stride1, p.k_stride2 = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
    p.v_stride0, p.v_stride1, p.v_stride2 = v_cache.stride(0), v_cache.stride(1), v_cache.stride(2)
    _lib.check(lib.jt_kv_store_launch(ctypes.byref(p), _launch.stream_handle(key.device)))

