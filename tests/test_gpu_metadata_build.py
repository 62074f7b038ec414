"""Device metadata builder: every field equal to the host builder's (itself pinned to the
reference's PackedTreeMetadata.build), and attention on it equal to attention on the host
build."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import PackedTreeMetadata, workloads

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
FIELDS = ("cu_seqlens_q", "query_to_request", "query_local_row", "prefix_lens",
          "block_tables", "tree_slots", "qq_bias", "qq_bias_offsets", "node_counts")


def _host_and_device(prefixes, tables, parents, arena, bs):
    total = sum(len(p) for p in parents)
    flat = [arena[j // bs] * bs + j % bs for j in range(total)]
    slots, cursor = [], 0
    for p in parents:
        slots.append(flat[cursor:cursor + len(p)])
        cursor += len(p)
    host = PackedTreeMetadata.from_parents(prefixes, tables, parents, slots, bs, device=DEV)
    dev = PackedTreeMetadata.from_parents_device(prefixes, tables, parents, arena, bs, device=DEV)
    torch.cuda.synchronize()
    return host, dev


def _assert_equal(host, dev):
    for name in FIELDS:
        a, b = getattr(host, name), getattr(dev, name)
        assert a.dtype == b.dtype and a.shape == b.shape, name
        assert torch.equal(a, b), name
    for name in ("prefix_lengths", "query_offsets", "node_counts_host", "block_tables_host",
                 "tree_slot_ids"):
        assert getattr(host, name) == getattr(dev, name), name


def test_ragged_batch_every_field():
    rng = np.random.default_rng(3)
    counts = [1, 5, 16, 33, 64, 128, 7]
    parents = [[-1] + [int(rng.integers(max(0, i - 8), i)) for i in range(1, n)] for n in counts]
    prefixes = [0, 1, 255, 256, 257, 1000, 4096]
    page = iter(range(10, 10_000))
    tables = [[next(page) for _ in range(-(-p // 256))] for p in prefixes]
    arena = [20_000 + i for i in range(3)]
    host, dev = _host_and_device(prefixes, tables, parents, arena, 256)
    _assert_equal(host, dev)
    assert jb.read_device_errors() == 0


def test_staged_topology_through_a_copy_stream():
    """The two public halves of from_parents_device as a pipelined caller uses them: the
    int32 topology in pinned memory, copied on a side stream, the device build on the
    compute stream after it; every field equals the host builder's."""
    batch = workloads.config3()
    used = {p for t in batch.block_tables for p in t}
    need = -(-batch.total_queries // 256)
    arena = [p for p in range(batch.num_blocks) if p not in used][:need]
    topo = PackedTreeMetadata.stage_topology(batch.prefix_lens, batch.block_tables,
                                             batch.parents, arena, 256)
    pinned = torch.from_numpy(topo.host).pin_memory()
    staged = torch.empty(pinned.shape, dtype=torch.int32, device=DEV)
    side = torch.cuda.Stream(DEV)
    with torch.cuda.stream(side):
        staged.copy_(pinned, non_blocking=True)
    torch.cuda.current_stream(DEV).wait_stream(side)
    dev = PackedTreeMetadata.from_staged_topology(staged, topo)
    host, _ = _host_and_device(batch.prefix_lens, batch.block_tables, batch.parents, arena, 256)
    _assert_equal(host, dev)
    with pytest.raises(ValueError, match="staged topology"):
        PackedTreeMetadata.from_staged_topology(staged[:-1], topo)


def test_largest_tree_and_deep_chain():
    parents = [[-1] + list(range(1023)), [-1] + [0] * 99]  # a 1024-deep chain, a wide star
    host, dev = _host_and_device([300, 5], [[1, 2], [3]], parents, [50 + i for i in range(5)], 256)
    _assert_equal(host, dev)


def test_attention_on_device_metadata_matches():
    batch = workloads.config2()
    q, k, v = workloads.make_tensors(batch, DEV, poison=False)  # every pool row finite
    used = {p for t in batch.block_tables for p in t}
    pages = [p for p in range(batch.num_blocks) if p not in used][:3]  # arena pages
    host, dev = _host_and_device(batch.prefix_lens, batch.block_tables, batch.parents, pages, 256)
    _assert_equal(host, dev)
    a = jb.packed_tree_attention_gqa(q, k, v, host, batch.head_dim ** -0.5, batch.groups)
    b = jb.packed_tree_attention_gqa(q, k, v, dev, batch.head_dim ** -0.5, batch.groups)
    torch.cuda.synchronize()
    assert torch.isfinite(a).all() and torch.equal(a, b)


def test_host_checks():
    with pytest.raises(ValueError, match="precede"):
        PackedTreeMetadata.from_parents_device([0], [[]], [[-1, 1]], [5], 256, device=DEV)
    with pytest.raises(ValueError, match="overlap"):
        PackedTreeMetadata.from_parents_device([10], [[5]], [[-1, 0]], [5], 256, device=DEV)
