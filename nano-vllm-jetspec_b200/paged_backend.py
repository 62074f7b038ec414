"""Tree-attention dispatcher with the reference's backend names.

Mirrors ``packed_tree_attention`` (nanovllm/speculative/jetspec/paged_backend.py:240-306).
Every backend runs the sm_100a kernel; they differ only in the probability arithmetic:

* ``"gqa"``  - probabilities rounded to the operand dtype before PV (the reference's
  opt-in grouped tensor-core contract, tree_gqa.py:105).
* ``"auto"``, ``"reference"``, ``"prefix"`` - near-fp32 probabilities in PV (hi + lo
  split of each probability), the reference's FP32-probability contract for these
  backends (paged_backend.py:1-7).  The reference's sm_120-only prefix specialisation
  has no separate meaning on B200.  These three also take fp32 q / k / v, as the
  reference's do (paged_backend.py:290-305, tree_attention.py:21-62): fp32 operands run
  on the CUDA-core fp32 kernel, every product, sum and softmax step in fp32.
"""
from __future__ import annotations

import torch

from .tree_gqa import _validate, launch_tree_attention, packed_tree_attention_gqa

BACKENDS = ("auto", "reference", "prefix", "gqa")


def packed_tree_attention(q, k_pool, v_pool, metadata, scale, num_queries_per_kv, *,
                          backend="auto", output_dtype=None):
    """One ragged launch with request-local prefix and ancestor visibility."""
    if backend not in BACKENDS:
        raise ValueError("tree attention backend must be auto, reference, prefix or gqa")
    if q.ndim != 3 or q.shape[0] != metadata.total_queries:
        raise ValueError("packed queries do not match the metadata")
    if k_pool.ndim != 4 or k_pool.shape != v_pool.shape or k_pool.shape[1] != metadata.block_size:
        raise ValueError("packed K/V page geometry does not match metadata")
    if (not q.is_cuda or q.device != k_pool.device or q.device != v_pool.device
            or q.device != metadata.tree_slots.device):
        raise ValueError("packed attention requires CUDA queries, KV and metadata on one device")
    _, num_query_heads, head_size = q.shape
    if q.stride(-1) != 1 or k_pool.shape[3] != head_size:
        raise ValueError("unsupported packed query/KV head geometry")
    if num_queries_per_kv <= 0 or num_query_heads != k_pool.shape[2] * num_queries_per_kv:
        raise ValueError("invalid packed GQA head grouping")
    if output_dtype not in (None, q.dtype, torch.float32):
        raise ValueError("output dtype must match input or be FP32 for qualification")
    if backend == "gqa":
        return packed_tree_attention_gqa(q, k_pool, v_pool, metadata, scale,
                                         num_queries_per_kv, output_dtype=output_dtype)
    out = _validate(q, k_pool, v_pool, metadata, num_queries_per_kv, output_dtype)
    return launch_tree_attention(out, q, k_pool, v_pool, metadata, scale, num_queries_per_kv,
                                 fp32_probability=True)


def packed_tree_attention_reference(q, k_pool, v_pool, metadata, scale, num_queries_per_kv,
                                    *, output_dtype=None):
    """FP32-probability entry (tree_attention.py:40-62 signature)."""
    return packed_tree_attention(q, k_pool, v_pool, metadata, scale, num_queries_per_kv,
                                 backend="reference", output_dtype=output_dtype)
