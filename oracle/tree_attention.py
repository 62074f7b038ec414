"""CPU restatement of the reference's tree-attention numerics (test infrastructure only).

masked_sdpa follows the reference's dense masked-SDPA seam:
  * prefix K/V gathered through the request's block table, position p at
    table[p // bs] * bs + p % bs   (nanovllm/layers/attention.py:87-93),
  * tree-node K/V appended from the request's scratch slots
    (nanovllm/speculative/jetspec/packed_metadata.py:185),
  * mask allowed = [ones(T, P) | ancestor(T, T)]
    (nanovllm/speculative/jetspec/runtime.py:486-488),
  * GQA expansion by repeat_interleave (nanovllm/models/qwen3.py:165-173),
  * F.scaled_dot_product_attention with a boolean mask and scale
    (nanovllm/models/qwen3.py:174-189), computed in fp32.

parent_chain_fp64 follows benchmarks/jetspec_numeric_oracles.py:72-105: one node's
query heads attend, unmasked, to the prefix followed by the node's root-to-node chain.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np
import torch
import torch.nn.functional as F


def ancestor_matrix(parents: Sequence[int]) -> np.ndarray:
    """Row j: node j and its ancestors (walks the parent chain of every node)."""
    count = len(parents)
    mask = np.zeros((count, count), dtype=bool)
    for node in range(count):
        current = node
        while current != -1:
            mask[node, current] = True
            current = int(parents[current])
    return mask


def parent_chain(parents: Sequence[int], node: int) -> list[int]:
    chain = []
    current = node
    while current != -1:
        chain.append(current)
        current = int(parents[current])
    return chain[::-1]


def _gather_rows(pool: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
    """Rows of `slots`, moved to the CPU (the pool itself may live on any device)."""
    block_size = pool.shape[1]
    slots = slots.to(pool.device)
    return pool[slots // block_size, slots % block_size].cpu()


def request_slots(prefix: int, table: Sequence[int], tree_slots: Sequence[int],
                  block_size: int) -> torch.Tensor:
    """Physical slots of a request's keys: prefix positions, then tree nodes."""
    positions = torch.arange(prefix, dtype=torch.int64)
    pages = torch.as_tensor(list(table), dtype=torch.int64)
    prefix_slots = (pages[positions // block_size] * block_size + positions % block_size
                    if prefix else torch.empty(0, dtype=torch.int64))
    return torch.cat((prefix_slots, torch.as_tensor(list(tree_slots), dtype=torch.int64)))


def masked_sdpa(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                prefix_lens: Sequence[int], block_tables: Sequence[Sequence[int]],
                tree_slots: Sequence[Sequence[int]], parents: Sequence[Sequence[int]],
                scale: float, groups: int, requests: Sequence[int] | None = None) -> torch.Tensor:
    """fp32 output [Q, Hq, D] of packed tree attention (rows of `requests` only).

    q [Q, Hq, D] and pools [blocks, bs, Hkv, D] may be of any float dtype (upcast to
    fp32) and on any device: only the request's rows are gathered and moved to the CPU,
    where all arithmetic runs.  Rows of requests not listed are left zero.
    """
    block_size = k_pool.shape[1]
    out = torch.zeros(q.shape, dtype=torch.float32)
    offsets = np.concatenate(([0], np.cumsum([len(p) for p in parents]))).astype(int)
    selected = range(len(prefix_lens)) if requests is None else requests
    for r in selected:
        prefix, nodes = int(prefix_lens[r]), len(parents[r])
        slots = request_slots(prefix, block_tables[r], tree_slots[r], block_size)
        keys = _gather_rows(k_pool, slots).float()
        values = _gather_rows(v_pool, slots).float()
        allowed = torch.ones((nodes, prefix + nodes), dtype=torch.bool)
        allowed[:, prefix:] = torch.from_numpy(ancestor_matrix(parents[r]))
        if groups > 1:
            keys = keys.repeat_interleave(groups, dim=1)
            values = values.repeat_interleave(groups, dim=1)
        rows = slice(offsets[r], offsets[r + 1])
        qh = q[rows].cpu().float().transpose(0, 1).unsqueeze(0)
        kh = keys.transpose(0, 1).unsqueeze(0)
        vh = values.transpose(0, 1).unsqueeze(0)
        result = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=allowed.view(1, 1, nodes, -1),
                                                dropout_p=0.0, scale=scale)
        out[rows] = result.squeeze(0).transpose(0, 1)
    return out


def parent_chain_fp64(q_row: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      prefix: int, table: Sequence[int], tree_slots: Sequence[int],
                      parents: Sequence[int], node: int, scale: float, groups: int) -> np.ndarray:
    """fp64 [Hq, D] attention of one node over its prefix and root-to-node chain."""
    block_size = k_pool.shape[1]
    chain = parent_chain(parents, node)
    slots = request_slots(prefix, table, [tree_slots[c] for c in chain], block_size)
    keys = _gather_rows(k_pool, slots).double().numpy()
    values = _gather_rows(v_pool, slots).double().numpy()
    query = q_row.cpu().double().numpy()
    out = np.zeros(query.shape, dtype=np.float64)
    for head in range(query.shape[0]):
        kv = head // groups
        scores = keys[:, kv] @ query[head] * scale
        scores -= scores.max()
        weights = np.exp(scores)
        weights /= weights.sum()
        out[head] = weights @ values[:, kv]
    return out
