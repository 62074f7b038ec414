"""Reference-facing Python API without a GPU: argument checks raise exactly where the
reference raises (tree_gqa.py:123-128, tree_attention.py:21-37, paged_backend.py:249-272,
attention.py:38-45, state.py:76-79), before any launch."""
from __future__ import annotations

import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import paged_backend, workloads
from jetspec_b200.attention import store_kvcache
from jetspec_b200.state import _slots_for_blocks, copy_accepted_kv


@pytest.fixture(scope="module")
def batch():
    return workloads.config1()


@pytest.fixture(scope="module")
def tensors(batch):
    q, k, v = workloads.make_tensors(batch, "cpu")
    return q, k, v, batch.metadata("cpu")


def test_gqa_argument_checks_in_reference_order(tensors):
    q, k, v, meta = tensors
    with pytest.raises(ValueError, match="query tile"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, 4, query_tile=2)
    with pytest.raises(ValueError, match="query tile"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, 4, query_tile=True)
    with pytest.raises(ValueError, match="BF16 or FP16"):
        jb.packed_tree_attention_gqa(q.float(), k, v, meta, 0.1, 4)
    with pytest.raises(ValueError, match="power-of-two"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, 3)
    with pytest.raises(ValueError, match="do not match the metadata"):
        jb.packed_tree_attention_gqa(q[:-1], k, v, meta, 0.1, 4)
    with pytest.raises(ValueError, match="page geometry"):
        jb.packed_tree_attention_gqa(q, k[:, :128], v[:, :128], meta, 0.1, 4)
    with pytest.raises(ValueError, match="CUDA"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, 4)


def test_dispatcher_checks(tensors):
    q, k, v, meta = tensors
    with pytest.raises(ValueError, match="backend"):
        paged_backend.packed_tree_attention(q, k, v, meta, 0.1, 4, backend="triton")
    with pytest.raises(ValueError, match="do not match the metadata"):
        paged_backend.packed_tree_attention(q[:-1], k, v, meta, 0.1, 4)
    # the device check precedes the grouping and output-dtype checks (paged_backend.py:265-272)
    with pytest.raises(ValueError, match="CUDA"):
        paged_backend.packed_tree_attention(q, k, v, meta, 0.1, 4, output_dtype=torch.float16)


def test_store_kvcache_layout_assertions():
    key = torch.zeros(4, 2, 8)
    cache = torch.zeros(3, 16, 2, 8)
    slots = torch.tensor([0, 1, -1, 5])
    with pytest.raises(AssertionError):
        store_kvcache(key.transpose(1, 2).contiguous().transpose(1, 2), key, cache, cache, slots)
    with pytest.raises(AssertionError):
        store_kvcache(key, key, cache.transpose(1, 2), cache, slots)
    with pytest.raises(AssertionError):
        store_kvcache(key, key, cache, cache, slots[:3])
    with pytest.raises(ValueError, match="CUDA"):
        store_kvcache(key, key, cache, cache, slots)


def test_copy_accepted_kv_checks_and_empty_commit():
    pool = torch.zeros(2, 1, 3, 16, 2, 8)
    with pytest.raises(ValueError, match="one-dimensional"):
        copy_accepted_kv(pool, torch.zeros(2, 2, dtype=torch.long), torch.zeros(4, dtype=torch.long), 16)
    with pytest.raises(ValueError, match="lengths differ"):
        copy_accepted_kv(pool, torch.zeros(3, dtype=torch.long), torch.zeros(4, dtype=torch.long), 16)
    assert copy_accepted_kv(pool, torch.zeros(0, dtype=torch.long),
                            torch.zeros(0, dtype=torch.long), 16) == 0
    with pytest.raises(ValueError, match="CUDA"):
        copy_accepted_kv(pool, torch.tensor([1]), torch.tensor([2]), 16)


def test_slots_for_blocks_mapping():
    slots = _slots_for_blocks([3, 0, 7], 5, 4, "cpu", start=6)
    assert slots.tolist() == [2, 3, 28, 29, 30]


def test_workloads_are_seeded_and_consistent():
    a, b = workloads.config3(), workloads.config3()
    assert a.prefix_lens == b.prefix_lens and a.parents == b.parents
    assert a.tree_slots == b.tree_slots and a.block_tables == b.block_tables
    assert a.num_requests == 64 and a.num_blocks == 16384
    keys = sum(p + t for p, t in zip(a.prefix_lens, a.node_counts))
    assert a.kv_bytes() == keys * 8 * 128 * 2 * 2
    live = a.live_slots()
    assert len(set(live.tolist())) == live.size  # prefixes and tree nodes never share a slot
    src, dst = a.commit_slots()
    assert len(src) == len(dst) == sum(len(p) for p in a.accepted_paths)
    c1 = workloads.config1()
    assert c1.prefix_lens == [512] and c1.block_tables == [[3, 0]] and c1.node_counts == [16]
    assert c1.commit_slots()[1] == [512, 513, 514, 515, 516]


def test_custom_operators_are_registered_with_fake_implementations():
    """The launchers are torch.library operators (what a torch.compile'd caller traces);
    their fake implementations accept meta tensors and write nothing."""
    import torch

    import jetspec_b200  # noqa: F401  (registers the operators)

    ops = torch.ops.jetspec_b200
    for name in ("tree_attention_", "kv_store_", "kv_commit_", "rope_scatter_"):
        assert hasattr(ops, name), name
    meta = torch.device("meta")
    out = torch.empty((8, 4, 128), device=meta)
    q = torch.empty((8, 4, 128), dtype=torch.bfloat16, device=meta)
    pool = torch.empty((4, 256, 1, 128), dtype=torch.bfloat16, device=meta)
    i32 = lambda n: torch.empty(n, dtype=torch.int32, device=meta)  # noqa: E731
    ops.tree_attention_(out, q, pool, pool, i32(2), i32(8), i32(8), i32(1), i32(1),
                        torch.empty((1, 1), dtype=torch.int32, device=meta),
                        torch.empty(8, dtype=torch.int64, device=meta),
                        torch.empty(64, device=meta), torch.empty(2, dtype=torch.int64, device=meta),
                        256, 0.1, 4, False, 0, False)
    kv = torch.empty((2, 1, 4, 256, 1, 128), dtype=torch.bfloat16, device=meta)
    ops.kv_commit_(kv, torch.empty(3, dtype=torch.int64, device=meta),
                   torch.empty(3, dtype=torch.int64, device=meta), 256)
    rows = torch.empty((8, 1, 128), dtype=torch.bfloat16, device=meta)
    ops.kv_store_(rows, rows, pool, pool, torch.empty(8, dtype=torch.int64, device=meta))
