"""Byte-level numpy restatement of the paged KV writes (test infrastructure only).

Arrays are raw element containers (bf16 travels as uint16); results must match the
kernels bit for bit.
"""
from __future__ import annotations

import numpy as np


def store_kvcache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray,
                  v_cache: np.ndarray, slot_mapping: np.ndarray) -> None:
    """In place: cache row `slot` of the flattened [blocks*bs, heads, dim] view gets row i.

    Follows store_kvcache_kernel (nanovllm/layers/attention.py:15-35): the cache is
    addressed as slot * (heads*dim) elements and slot == -1 is skipped.
    """
    k_rows = k_cache.reshape(-1, *k_cache.shape[2:])
    v_rows = v_cache.reshape(-1, *v_cache.shape[2:])
    for i, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot == -1:
            continue
        k_rows[slot] = key[i]
        v_rows[slot] = value[i]


def copy_accepted_kv(kv_pool: np.ndarray, source_slots: np.ndarray,
                     destination_slots: np.ndarray, block_size: int) -> int:
    """In place on a [2, L, blocks, bs, Hkv, D] pool; returns payload bytes.

    Follows copy_accepted_kv (nanovllm/speculative/jetspec/state.py:64-86): the selected
    rows are materialised before the scatter, so overlapping slot sets are safe.
    """
    src = np.asarray(source_slots, dtype=np.int64)
    dst = np.asarray(destination_slots, dtype=np.int64)
    if src.ndim != 1 or dst.ndim != 1:
        raise ValueError("KV copy requires one-dimensional slot maps")
    if src.size != dst.size:
        raise ValueError("KV copy source and destination lengths differ")
    accepted = kv_pool[:, :, src // block_size, src % block_size].copy()
    kv_pool[:, :, dst // block_size, dst % block_size] = accepted
    return int(accepted.size * accepted.itemsize)
