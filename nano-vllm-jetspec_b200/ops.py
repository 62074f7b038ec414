"""torch.library registration of the launchers (the custom-op half of the boundary).

The Python wrappers call the C ABI through ctypes, which a tracing compiler cannot see
into: a ``torch.compile``d caller (the reference compiles its norms and rotary embedding,
nanovllm/layers/layernorm.py, rotary_embedding.py) would break its graph at every kernel.
Each launcher is therefore also a custom operator in the ``jetspec_b200`` namespace, with
a fake (shape-only) implementation, and the public wrappers route through it while
``torch.compiler.is_compiling()``; eager calls keep the direct launch (no dispatcher
overhead).  The operators mutate their output arguments in place and return nothing, so
functionalisation sees exactly which buffers they write.

* ``jetspec_b200::tree_attention_`` - out[Q, Hq, D] <- packed tree attention
* ``jetspec_b200::kv_store_``       - k_cache / v_cache rows <- key / value
* ``jetspec_b200::kv_commit_``      - kv_pool accepted rows moved to their destinations
* ``jetspec_b200::rope_scatter_``   - out <- rope(q); k_pool / v_pool <- rope(k) / v
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

NAMESPACE = "jetspec_b200"


@torch.library.custom_op(f"{NAMESPACE}::tree_attention_", mutates_args=("out",))
def tree_attention_(out: torch.Tensor, q: torch.Tensor, k_pool: torch.Tensor,
                    v_pool: torch.Tensor, cu_seqlens_q: torch.Tensor,
                    query_to_request: torch.Tensor, query_local_row: torch.Tensor,
                    prefix_lens: torch.Tensor, node_counts: torch.Tensor,
                    block_tables: torch.Tensor, tree_slots: torch.Tensor, qq_bias: torch.Tensor,
                    qq_bias_offsets: torch.Tensor, block_size: int, scale: float, groups: int,
                    fp32_probability: bool, split_keys: int, portable_core: bool) -> None:
    from .tree_gqa import launch_tree_attention_eager

    metadata = SimpleNamespace(
        cu_seqlens_q=cu_seqlens_q, query_to_request=query_to_request,
        query_local_row=query_local_row, prefix_lens=prefix_lens, node_counts=node_counts,
        block_tables=block_tables, tree_slots=tree_slots, qq_bias=qq_bias,
        qq_bias_offsets=qq_bias_offsets, block_size=block_size,
        num_requests=int(prefix_lens.numel()), total_queries=int(q.shape[0]),
        node_counts_host=None)
    launch_tree_attention_eager(out, q, k_pool, v_pool, metadata, scale, groups,
                                fp32_probability=fp32_probability, split_keys=split_keys,
                                portable_core=portable_core)


@tree_attention_.register_fake
def _(out, q, k_pool, v_pool, cu_seqlens_q, query_to_request, query_local_row, prefix_lens,
      node_counts, block_tables, tree_slots, qq_bias, qq_bias_offsets, block_size, scale,
      groups, fp32_probability, split_keys, portable_core):
    return None


@torch.library.custom_op(f"{NAMESPACE}::kv_store_", mutates_args=("k_cache", "v_cache"))
def kv_store_(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
              v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    from .attention import _store

    _store(key, value, k_cache, v_cache, slot_mapping)


@kv_store_.register_fake
def _(key, value, k_cache, v_cache, slot_mapping):
    return None


@torch.library.custom_op(f"{NAMESPACE}::kv_commit_", mutates_args=("kv_pool",))
def kv_commit_(kv_pool: torch.Tensor, source_slots: torch.Tensor,
               destination_slots: torch.Tensor, block_size: int) -> None:
    from .state import _commit

    _commit(kv_pool, source_slots, destination_slots, block_size)


@kv_commit_.register_fake
def _(kv_pool, source_slots, destination_slots, block_size):
    return None


@torch.library.custom_op(f"{NAMESPACE}::rope_scatter_",
                         mutates_args=("k_pool", "v_pool", "out"))
def rope_scatter_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
                  cos_sin_cache: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                  node_slots: torch.Tensor, out: torch.Tensor) -> None:
    from .tree_fusion import _rope_scatter_launch

    _rope_scatter_launch(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots, out)


@rope_scatter_.register_fake
def _(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots, out):
    return None


def compiling() -> bool:
    """True while torch.compile traces the caller (route through the operators)."""
    return torch.compiler.is_compiling()
