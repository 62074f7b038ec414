"""CPU restatement of the fused HF-order RoPE + node K/V scatter (test infrastructure only).

eager_rope follows the reference's eager definition (tests/test_jetspec_tree_fusion.py:21-32,
the contract of nanovllm/speculative/jetspec/tree_fusion.py:20-28): cos / sin are the two
halves of the cache row at each position, converted to the operand dtype; every product
is rounded to the operand dtype before the add / subtract (PyTorch eager arithmetic on
bf16 tensors).  rope_scatter applies it to Q (returned) and K (written to the node slots
of the K pool) and copies V to the same slots.
"""
from __future__ import annotations

import torch


def eager_rope(x: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor) -> torch.Tensor:
    selected = cache[positions.long().cpu()]
    if selected.ndim == 2:
        selected = selected.unsqueeze(1)
    cos, sin = selected.chunk(2, -1)
    cos, sin = cos.to(x.dtype), sin.to(x.dtype)
    x1, x2 = x.chunk(2, -1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1)


def rope_scatter(q, k, v, positions, cache, k_pool, v_pool, node_slots):
    """In place on CPU pools; returns the rotated Q."""
    q, k, v, cache = q.cpu(), k.cpu(), v.cpu(), cache.cpu()
    slots = node_slots.long().cpu()
    page_size = k_pool.shape[1]
    k_pool[slots // page_size, slots % page_size] = eager_rope(k, positions, cache)
    v_pool[slots // page_size, slots % page_size] = v
    return eager_rope(q, positions, cache)
