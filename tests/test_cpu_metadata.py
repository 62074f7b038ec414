"""PackedTreeMetadata: golden equality with the reference builder and its CPU gates.

Mirrors tests/test_jetspec_packed_attention.py:47-101 of the reference (metadata offsets,
tables, rejection of overlapping / committed scratch pages, non-canonical tables and
malformed ancestor masks, pool geometry checks).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_cases import load_npz
from jetspec_b200.packed_metadata import PackedTreeMetadata, ancestor_mask_from_parents


def heap_ancestors(nodes):
    result = torch.zeros((nodes, nodes), dtype=torch.bool)
    for node in range(nodes):
        current = node
        while current >= 0:
            result[node, current] = True
            current = (current - 1) // 2
    return result


def fixture(counts=(63, 31, 47)):
    starts = np.concatenate(([0], np.cumsum(counts))).astype(int)
    slots = [torch.arange(6 * 256 + starts[i], 6 * 256 + starts[i + 1], dtype=torch.int64)
             for i in range(len(counts))]
    prefixes = (65, 0, 257)[:len(counts)]
    pages = ((2,), (), (4, 0))[:len(counts)]
    masks = [heap_ancestors(c) for c in counts]
    return PackedTreeMetadata.build(prefixes, pages, slots, masks, 256), slots, masks


def test_device_buffers_equal_reference_builder():
    meta, _, _ = fixture()
    z = load_npz("metadata_ragged3.npz")
    for name in ("cu_seqlens_q", "query_to_request", "query_local_row", "prefix_lens",
                 "block_tables", "tree_slots", "qq_bias_offsets", "node_counts"):
        got = getattr(meta, name)
        assert got.dtype == torch.from_numpy(z[name]).dtype, name
        assert np.array_equal(got.numpy(), z[name]), name
    bias = meta.qq_bias.numpy()
    assert bias.dtype == z["qq_bias"].dtype
    assert np.array_equal(np.isneginf(bias), np.isneginf(z["qq_bias"]))
    assert np.array_equal(bias[np.isfinite(bias)], z["qq_bias"][np.isfinite(z["qq_bias"])])


def test_exact_ragged_offsets_and_local_masks():
    meta, _, _ = fixture()
    assert meta.query_offsets == (0, 63, 94, 141)
    assert meta.request_slice(1) == slice(63, 94)
    assert meta.prefix_lengths == (65, 0, 257)
    assert meta.node_counts_host == (63, 31, 47)
    assert meta.mask_elements == 63 ** 2 + 31 ** 2 + 47 ** 2
    assert meta.block_tables.tolist() == [[2, -1], [-1, -1], [4, 0]]
    assert meta.query_to_request.tolist() == [0] * 63 + [1] * 31 + [2] * 47
    assert meta.query_local_row.tolist() == list(range(63)) + list(range(31)) + list(range(47))
    assert meta.report()["numerical_contract"] == "fp32_online_softmax_tile64"
    with pytest.raises(IndexError):
        meta.request_slice(-1)
    with pytest.raises(IndexError):
        meta.request_slice(3)


def test_rejects_overlapping_scratch_and_committed_pages():
    _, slots, masks = fixture()
    with pytest.raises(ValueError, match="overlapping"):
        PackedTreeMetadata.build([65, 0], [[2], []], [slots[0], slots[0][:31]], masks[:2], 256)
    with pytest.raises(ValueError, match="committed"):
        PackedTreeMetadata.build([65], [[6]], [slots[0]], masks[:1], 256)


def test_rejects_noncanonical_tables_and_malformed_ancestors():
    _, slots, masks = fixture()
    with pytest.raises(ValueError, match="canonical"):
        PackedTreeMetadata.build([257], [[2]], slots[:1], masks[:1], 256)
    with pytest.raises(ValueError, match="canonical"):
        PackedTreeMetadata.build([257], [[2, 2]], slots[:1], masks[:1], 256)
    future = masks[0].clone()
    future[0, 1] = True
    with pytest.raises(ValueError, match="causal"):
        PackedTreeMetadata.build([65], [[2]], slots[:1], [future], 256)
    missing_self = masks[0].clone()
    missing_self[1, 1] = False
    with pytest.raises(ValueError, match="self"):
        PackedTreeMetadata.build([65], [[2]], slots[:1], [missing_self], 256)


def test_pool_bounds_and_geometry():
    meta, _, _ = fixture()
    meta.validate_pool_geometry(torch.empty(2, 3, 8, 256, 2, 4))
    with pytest.raises(ValueError, match="geometry"):
        meta.validate_pool_geometry(torch.empty(2, 3, 8, 16, 2, 4))
    with pytest.raises(ValueError, match="outside"):
        meta.validate_pool_geometry(torch.empty(2, 3, 6, 256, 2, 4))


def test_from_parents_equals_build_with_ancestor_masks():
    rng = np.random.default_rng(5)
    parents = [[-1] + [int(rng.integers(0, i)) for i in range(1, n)] for n in (9, 4, 17)]
    starts = np.concatenate(([0], np.cumsum([len(p) for p in parents]))).astype(int)
    slots = [list(range(5 * 256 + starts[i], 5 * 256 + starts[i + 1])) for i in range(3)]
    prefixes, tables = (300, 0, 12), ((1, 3), (), (0,))
    a = PackedTreeMetadata.from_parents(prefixes, tables, parents, slots, 256, device="cpu")
    masks = [torch.from_numpy(ancestor_mask_from_parents(p)) for p in parents]
    b = PackedTreeMetadata.build(prefixes, tables,
                                 [torch.tensor(s, dtype=torch.int64) for s in slots], masks, 256)
    for name in ("cu_seqlens_q", "query_to_request", "query_local_row", "prefix_lens",
                 "block_tables", "tree_slots", "qq_bias", "qq_bias_offsets", "node_counts"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
