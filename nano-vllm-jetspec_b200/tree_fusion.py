"""Tree-node KV write into scratch slots before verification.

``scatter_tree_kv`` is the non-fused node write of the verifier
(nanovllm/models/qwen3.py:255-258: ``k_pool[slot // bs, slot % bs] = k`` and the same
for V) as one launch of the warp-per-token store kernel.
"""
from __future__ import annotations

import torch

from .attention import _store


def scatter_tree_kv(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                    v_pool: torch.Tensor, node_slots: torch.Tensor) -> None:
    """Write node K/V rows [Q, kv_heads, dim] to their scratch slots (bit-exact)."""
    if k.ndim != 3 or v.shape != k.shape or node_slots.shape != (k.shape[0],):
        raise ValueError("node K/V must be [rows, kv_heads, dim] with one slot per row")
    _store(k, v, k_pool, v_pool, node_slots.contiguous())
