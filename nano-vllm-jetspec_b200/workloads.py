"""Seeded synthetic tree-verification batches with the benchmark configurations' shapes.

There is no serving trace or checkpoint here, so every input is synthetic: random-parent
trees in topological order, prefix pages drawn from a shuffled physical pool, tree nodes
at scattered scratch slots of pages no prefix owns, q/k/v ~ N(0, 1)/sqrt(head_dim), and
accepted root-to-node paths for the commit.  Unleased pool rows can be poisoned with NaN
so that any out-of-bounds read shows up as a non-finite output.
"""
from __future__ import annotations

from dataclasses import dataclass, field
import math

import numpy as np
import torch

from .packed_metadata import PackedTreeMetadata


@dataclass
class TreeBatch:
    prefix_lens: list[int]
    parents: list[list[int]]
    block_tables: list[list[int]]   # tight prefix tables (what attention reads)
    owned_pages: list[list[int]]    # prefix pages + headroom for the accepted commit
    tree_slots: list[list[int]]
    accepted_paths: list[list[int]]
    num_blocks: int
    block_size: int = 256
    num_kv_heads: int = 8
    groups: int = 4
    head_dim: int = 128
    seed: int = 0
    name: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def num_requests(self) -> int:
        return len(self.prefix_lens)

    @property
    def node_counts(self) -> list[int]:
        return [len(p) for p in self.parents]

    @property
    def total_queries(self) -> int:
        return sum(self.node_counts)

    @property
    def num_query_heads(self) -> int:
        return self.num_kv_heads * self.groups

    def metadata(self, device) -> PackedTreeMetadata:
        return PackedTreeMetadata.from_parents(self.prefix_lens, self.block_tables, self.parents,
                                               self.tree_slots, self.block_size, device=device)

    def kv_bytes(self, kv_heads: int | None = None, elem_bytes: int = 2) -> int:
        """K+V bytes the attention reads: sum_r (P_r + T_r) * heads * dim * 2 tensors."""
        heads = self.num_kv_heads if kv_heads is None else kv_heads
        keys = sum(p + t for p, t in zip(self.prefix_lens, self.node_counts))
        return keys * heads * self.head_dim * elem_bytes * 2

    def attention_flops(self, kv_heads: int | None = None) -> int:
        """4*D flops per visible (query head, key) pair: QK^T and PV."""
        heads = self.num_kv_heads if kv_heads is None else kv_heads
        pairs = 0
        for prefix, parents in zip(self.prefix_lens, self.parents):
            depths = _depths(parents)
            pairs += len(parents) * prefix + sum(d + 1 for d in depths)
        return pairs * heads * self.groups * 4 * self.head_dim

    def commit_slots(self) -> tuple[list[int], list[int]]:
        """(source, destination) slots of every accepted node, request after request."""
        src, dst = [], []
        for prefix, pages, slots, path in zip(self.prefix_lens, self.owned_pages,
                                              self.tree_slots, self.accepted_paths):
            for i, node in enumerate(path):
                pos = prefix + i
                src.append(slots[node])
                dst.append(pages[pos // self.block_size] * self.block_size + pos % self.block_size)
        return src, dst

    def live_slots(self) -> np.ndarray:
        """Every physical slot holding valid K/V: prefixes and tree nodes."""
        chunks = []
        for prefix, table, slots in zip(self.prefix_lens, self.block_tables, self.tree_slots):
            pos = np.arange(prefix, dtype=np.int64)
            pages = np.asarray(table, dtype=np.int64)
            if prefix:
                chunks.append(pages[pos // self.block_size] * self.block_size + pos % self.block_size)
            chunks.append(np.asarray(slots, dtype=np.int64))
        return np.concatenate(chunks)


def _depths(parents) -> list[int]:
    depths = [0] * len(parents)
    for node in range(1, len(parents)):
        depths[node] = depths[parents[node]] + 1
    return depths


def random_parents(rng: np.random.Generator, nodes: int, window: int | None = None) -> list[int]:
    """parent(i) uniform in [max(0, i - window), i - 1] (window None: [0, i - 1])."""
    parents = [-1]
    for node in range(1, nodes):
        low = 0 if window is None else max(0, node - window)
        parents.append(int(rng.integers(low, node)))
    return parents


def _deepest_chain(parents) -> list[int]:
    depths = _depths(parents)
    node = int(np.argmax(depths))
    chain = []
    while node != -1:
        chain.append(node)
        node = parents[node]
    return chain[::-1]


def build_batch(prefix_lens, parents, *, num_blocks=None, block_size=256, num_kv_heads=8,
                groups=4, head_dim=128, seed=0, accepted_lengths=None, scatter_slots=True,
                headroom_pages=1, name="") -> TreeBatch:
    """Random physical layout for the given prefixes and trees.

    Prefix pages and scratch pages come from one shuffled page list, so prefixes are
    non-contiguous and no scratch page is shared with a prefix; tree slots are a random
    permutation of the scratch slots unless ``scatter_slots`` is False.
    """
    rng = np.random.default_rng(seed)
    prefix_lens = [int(p) for p in prefix_lens]
    counts = [len(p) for p in parents]
    if accepted_lengths is None:
        accepted_lengths = [min(len(_deepest_chain(p)), 1) for p in parents]
    paths = []
    for tree, length in zip(parents, accepted_lengths):
        chain = _deepest_chain(tree)
        paths.append(chain[:max(1, min(int(length), len(chain)))])
    owned_counts = [-(-(p + len(path)) // block_size) + headroom_pages
                    for p, path in zip(prefix_lens, paths)]
    scratch_pages = -(-sum(counts) // block_size) + 1
    needed = sum(owned_counts) + scratch_pages
    if num_blocks is None:
        num_blocks = needed + 3
    if num_blocks < needed:
        raise ValueError(f"pool of {num_blocks} pages cannot hold {needed} pages")
    order = rng.permutation(num_blocks).tolist()
    cursor = 0
    owned, tables = [], []
    for prefix, count in zip(prefix_lens, owned_counts):
        pages = order[cursor:cursor + count]
        cursor += count
        owned.append(pages)
        tables.append(pages[:-(-prefix // block_size)] if prefix else [])
    scratch = order[cursor:cursor + scratch_pages]
    slots = np.asarray([page * block_size + off for page in scratch for off in range(block_size)],
                       dtype=np.int64)
    if scatter_slots:
        slots = slots[rng.permutation(slots.size)]
    tree_slots, cursor = [], 0
    for count in counts:
        tree_slots.append(slots[cursor:cursor + count].tolist())
        cursor += count
    return TreeBatch(prefix_lens, [list(p) for p in parents], tables, owned, tree_slots, paths,
                     num_blocks, block_size, num_kv_heads, groups, head_dim, seed, name)


def make_tensors(batch: TreeBatch, device, dtype=torch.bfloat16, *, poison=True,
                 std=None, generator_device="cpu"):
    """(q, k_pool, v_pool): live rows ~ N(0, std^2) (default 1/sqrt(head_dim)); others NaN."""
    std = batch.head_dim ** -0.5 if std is None else std
    gen = torch.Generator(device=generator_device).manual_seed(batch.seed + 7)
    Q, Hq, D = batch.total_queries, batch.num_query_heads, batch.head_dim
    q = (torch.randn((Q, Hq, D), generator=gen, device=generator_device) * std).to(dtype)
    shape = (batch.num_blocks, batch.block_size, batch.num_kv_heads, D)
    live = torch.from_numpy(batch.live_slots())
    pools = []
    for _ in range(2):
        if poison:
            pool = torch.full(shape, float("nan"), dtype=dtype, device=device)
            rows = (torch.randn((live.numel(), batch.num_kv_heads, D), generator=gen,
                                device=generator_device) * std).to(dtype).to(device)
            flat = pool.view(-1, batch.num_kv_heads, D)
            flat[live.to(device)] = rows
        else:
            pool = (torch.randn(shape, generator=gen, device=generator_device) * std).to(dtype)
            pool = pool.to(device)
        pools.append(pool)
    return q.to(device), pools[0], pools[1]


# ---- the benchmark configurations -------------------------------------------------------
def config1(seed=1001) -> TreeBatch:
    """1 request, prefix 512 on pages [3, 0], 16-node random-parent tree on page 4,
    5-node accepted path committed to slots 512-516 (page 2)."""
    rng = np.random.default_rng(seed)
    parents = random_parents(rng, 16)
    chain = _deepest_chain(parents)
    path = chain[:5]
    slots = [4 * 256 + i for i in range(16)]
    return TreeBatch([512], [parents], [[3, 0]], [[3, 0, 2]], [slots], [path], 5,
                     seed=seed, name="config1")


def config2(seed=1002) -> TreeBatch:
    """8 requests, prefixes U[1024, 4096], 64-node trees (parent in [i-8, i-1]),
    2048-page shuffled pool."""
    rng = np.random.default_rng(seed)
    prefixes = rng.integers(1024, 4097, size=8).tolist()
    parents = [random_parents(rng, 64, window=8) for _ in range(8)]
    accepted = _geometric(rng, parents, 0.35)
    return build_batch(prefixes, parents, num_blocks=2048, seed=seed, accepted_lengths=accepted,
                       name="config2")


def config3(seed=1003, num_requests=64, num_blocks=None) -> TreeBatch:
    """Serving mix: 64 requests, context log-uniform [512, 16384], tree budgets from
    {16, 32, 64, 128}, accepted lengths Geometric(0.35) capped at the tree depth,
    shuffled pool of 16384 pages per 64 requests (``num_blocks`` overrides it)."""
    rng = np.random.default_rng(seed)
    prefixes = np.exp(rng.uniform(math.log(512), math.log(16384), size=num_requests))
    prefixes = prefixes.astype(np.int64).tolist()
    budgets = rng.choice([16, 32, 64, 128], size=num_requests).tolist()
    parents = [random_parents(rng, int(t), window=8) for t in budgets]
    accepted = _geometric(rng, parents, 0.35)
    if num_blocks is None:
        num_blocks = 16384 * max(1, -(-num_requests // 64))
    return build_batch(prefixes, parents, num_blocks=num_blocks, seed=seed,
                       accepted_lengths=accepted, name="config3")


def config4(seed=1004, num_kv_heads=8) -> TreeBatch:
    """Long context: 16 requests x 32768-token prefixes, 64-node trees."""
    rng = np.random.default_rng(seed)
    parents = [random_parents(rng, 64, window=8) for _ in range(16)]
    accepted = _geometric(rng, parents, 0.35)
    return build_batch([32768] * 16, parents, seed=seed, accepted_lengths=accepted,
                       num_kv_heads=num_kv_heads, name="config4")


def _geometric(rng, parents, p):
    out = []
    for tree in parents:
        cap = len(_deepest_chain(tree))
        out.append(int(min(rng.geometric(p), cap)))
    return out


CONFIGS = {"config1": config1, "config2": config2, "config3": config3, "config4": config4}
