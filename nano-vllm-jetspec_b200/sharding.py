"""KV-head sharding of tree verification across the GPUs of one node.

Every (request, KV head) pair is independent, so the path shards by KV-head group with
no data exchange inside attention: rank g of N owns KV heads [g*Hkv/N, (g+1)*Hkv/N) and
the query heads that read them, the same split as the reference's tensor-parallel head
partition (nanovllm/models/qwen3.py:39-45, nanovllm/engine/model_runner.py:110).
Packed metadata (tables, slots, ancestor bias) is replicated on every rank, and the
store / commit kernels run per shard with identical slot lists.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class KvHeadShard:
    rank: int
    world_size: int
    num_kv_heads: int
    groups: int

    @property
    def local_kv_heads(self) -> int:
        return self.num_kv_heads // self.world_size

    @property
    def kv_head_begin(self) -> int:
        return self.rank * self.local_kv_heads

    @property
    def kv_head_end(self) -> int:
        return self.kv_head_begin + self.local_kv_heads

    @property
    def q_head_begin(self) -> int:
        return self.kv_head_begin * self.groups

    @property
    def q_head_end(self) -> int:
        return self.kv_head_end * self.groups

    def slice_queries(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of packed [Q, q_heads, dim] rows (a view)."""
        return q[:, self.q_head_begin:self.q_head_end]

    def slice_pool(self, pool: torch.Tensor) -> torch.Tensor:
        """This rank's heads of a [blocks, bs, kv_heads, dim] pool (a view)."""
        return pool[:, :, self.kv_head_begin:self.kv_head_end]

    def slice_kv_rows(self, rows: torch.Tensor) -> torch.Tensor:
        """This rank's heads of [N, kv_heads, dim] K or V rows (a view)."""
        return rows[:, self.kv_head_begin:self.kv_head_end]


def shard_for_rank(num_kv_heads: int, groups: int, world_size: int, rank: int) -> KvHeadShard:
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    if num_kv_heads % world_size:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world_size} ranks")
    if groups < 1:
        raise ValueError("groups must be positive")
    return KvHeadShard(rank, world_size, num_kv_heads, groups)
