"""Accepted-only KV commit: drop-in for ``copy_accepted_kv``.

Same signature, return value and ValueError behaviour as
nanovllm/speculative/jetspec/state.py:64-86.  The copy runs as one cooperative sm_100a
kernel spread over the whole GPU; every source row of a (K/V axis, layer) plane is read
before any row of that plane is written (a grid barrier between the gather and the
scatter), so overlapping source/destination slot sets give the same bytes as the
reference's materialised advanced-index copy.
"""
from __future__ import annotations

import ctypes

import torch

from . import _launch, _lib


def _slots_for_blocks(blocks, length, block_size, device, *, start=0):
    """Physical slots of logical positions [start, start+length) through a page list.

    Same mapping as the reference helper (state.py:54-61).
    """
    table = torch.tensor(list(blocks), dtype=torch.long, device=device)
    positions = torch.arange(start, start + length, dtype=torch.long, device=device)
    return table[positions // block_size] * block_size + positions % block_size


def copy_accepted_kv(kv_pool: torch.Tensor, source_slots: torch.Tensor,
                     destination_slots: torch.Tensor, block_size: int) -> int:
    """Copy accepted post-RoPE K/V rows across both KV axes and all layers.

    Returns the payload size in bytes (slots x 2 x layers x kv_heads x head_dim x
    element size), not the read + write traffic.
    """
    if source_slots.ndim != 1 or destination_slots.ndim != 1:
        raise ValueError("KV copy requires one-dimensional slot maps")
    if source_slots.numel() != destination_slots.numel():
        raise ValueError("KV copy source and destination lengths differ")
    if kv_pool.ndim != 6 or kv_pool.shape[0] != 2 or kv_pool.shape[3] != int(block_size):
        raise ValueError("KV pool must be [2, layers, blocks, block_size, kv_heads, head_dim]")
    n = int(source_slots.numel())
    payload = n * 2 * int(kv_pool.shape[1]) * int(kv_pool.shape[4]) * int(kv_pool.shape[5]) \
        * kv_pool.element_size()
    if n == 0:
        return 0
    if not kv_pool.is_cuda or source_slots.device != kv_pool.device \
            or destination_slots.device != kv_pool.device:
        raise ValueError("KV commit requires the pool and slot maps on one CUDA device")
    if source_slots.dtype not in (torch.int32, torch.int64):
        raise ValueError("slot maps must be int32 or int64")
    if destination_slots.dtype != source_slots.dtype:
        destination_slots = destination_slots.to(source_slots.dtype)
    source_slots = source_slots.contiguous()
    destination_slots = destination_slots.contiguous()
    if kv_pool.stride(-1) != 1:
        raise ValueError("KV pool needs a contiguous head dimension")
    from . import ops

    if ops.compiling():
        torch.ops.jetspec_b200.kv_commit_(kv_pool, source_slots, destination_slots, int(block_size))
    else:
        _commit(kv_pool, source_slots, destination_slots, block_size)
    return int(payload)


def _commit(kv_pool, source_slots, destination_slots, block_size) -> None:
    """jt_kv_commit_launch on the current stream (validated arguments)."""
    lib = _lib.load_library()
    n = int(source_slots.numel())
    if n > lib.jt_kv_commit_max_slots():
        raise ValueError(f"KV commit of {n} slots exceeds the per-call limit "
                         f"{lib.jt_kv_commit_max_slots()}")
    p = _lib.JtKvCommitParams()
    p.kv_pool = kv_pool.data_ptr()
    p.source_slots = source_slots.data_ptr()
    p.destination_slots = destination_slots.data_ptr()
    p.slot_is_int64 = int(source_slots.dtype == torch.int64)
    p.num_slots = n
    p.num_layers = int(kv_pool.shape[1])
    p.num_kv_heads = int(kv_pool.shape[4])
    p.head_dim = int(kv_pool.shape[5])
    p.elem_bytes = kv_pool.element_size()
    p.block_size = int(block_size)
    p.num_blocks = int(kv_pool.shape[2])
    s = kv_pool.stride()
    p.stride_axis, p.stride_layer, p.stride_block, p.stride_offset, p.stride_head = \
        s[0], s[1], s[2], s[3], s[4]
    _lib.check(lib.jt_kv_commit_launch(ctypes.byref(p), _launch.stream_handle(kv_pool.device)))
