"""The CPU oracle pinned to the reference's own outputs (golden fixtures; no GPU).

The fixtures come from running the reference's fp32 tree-attention kernel
(paged_backend.py _packed_paged_tree_fp32) under the Triton interpreter, its fp64
parent-chain oracle (benchmarks/jetspec_numeric_oracles.py), its store_kvcache kernel
(layers/attention.py) and its copy_accepted_kv (speculative/jetspec/state.py).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_cases import load_attn_case, load_npz
from oracle import kv_cache as kv_oracle
from oracle import tree_attention as attn_oracle

CASES = ("ragged3", "config1")


def _oracle(case):
    return attn_oracle.masked_sdpa(case.q, case.k_pool, case.v_pool, case.prefixes, case.tables,
                                   case.tree_slots, case.parents, case.scale, case.groups)


@pytest.mark.parametrize("name", CASES)
def test_masked_sdpa_matches_reference_fp32_kernel(name):
    case = load_attn_case(name)
    out = _oracle(case)
    assert torch.isfinite(out).all(), "oracle read a poisoned (unleased) row"
    diff = (out - case.ref_out).abs().max().item()
    assert diff <= 2e-6, f"oracle vs reference fp32 kernel: max-abs {diff:.3e}"


@pytest.mark.parametrize("name", CASES)
def test_parent_chain_fp64_matches_reference_fp64_oracle(name):
    case = load_attn_case(name)
    offsets = np.concatenate(([0], np.cumsum([len(p) for p in case.parents])))
    for row, expected in zip(case.fp64_rows, case.fp64_out):
        r = int(np.searchsorted(offsets, row, side="right") - 1)
        node = int(row - offsets[r])
        got = attn_oracle.parent_chain_fp64(case.q[row], case.k_pool, case.v_pool,
                                            case.prefixes[r], case.tables[r], case.tree_slots[r],
                                            case.parents[r], node, case.scale, case.groups)
        np.testing.assert_allclose(got, expected, rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", CASES)
def test_reference_fp32_kernel_agrees_with_its_fp64_oracle(name):
    """The golden itself: fp32 kernel rows within the reference's 1e-4 fp32 bound."""
    case = load_attn_case(name)
    got = case.ref_out[torch.from_numpy(case.fp64_rows)].double().numpy()
    assert np.abs(got - case.fp64_out).max() <= 1e-4


def test_ancestor_matrix_and_parent_chain():
    parents = [-1, 0, 0, 1, 2, 3]
    assert attn_oracle.parent_chain(parents, 5) == [0, 1, 3, 5]
    mask = attn_oracle.ancestor_matrix(parents)
    assert mask.diagonal().all() and not np.triu(mask, 1).any()
    assert mask[5].nonzero()[0].tolist() == [0, 1, 3, 5]
    assert mask[4].nonzero()[0].tolist() == [0, 2, 4]


def test_store_kvcache_oracle_matches_reference():
    z = load_npz("kv_store.npz")
    k, v = z["k_before"].copy(), z["v_before"].copy()
    kv_oracle.store_kvcache(z["key"], z["value"], k, v, z["slots"])
    assert np.array_equal(k.view(np.uint32), z["k_after"].view(np.uint32))
    assert np.array_equal(v.view(np.uint32), z["v_after"].view(np.uint32))


def test_copy_accepted_kv_oracle_matches_reference():
    z = load_npz("kv_commit.npz")
    pool = z["before"].copy()
    nbytes = kv_oracle.copy_accepted_kv(pool, z["src"], z["dst"], 16)
    assert nbytes == int(z["nbytes"])
    assert np.array_equal(pool.view(np.uint32), z["after"].view(np.uint32))
