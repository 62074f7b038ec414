"""CUDA path against the reference's own outputs (golden fixtures from tests/golden/)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import paged_backend
from jetspec_b200.attention import store_kvcache
from jetspec_b200.packed_metadata import PackedTreeMetadata
from jetspec_b200.state import copy_accepted_kv

from golden_cases import load_attn_case, load_npz
from helpers import FP32_BOUND, assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _inputs(case):
    meta = PackedTreeMetadata.from_parents(case.prefixes, case.tables, case.parents,
                                           case.tree_slots, 256, device=DEV)
    return case.q.to(DEV), case.k_pool.to(DEV), case.v_pool.to(DEV), meta


def test_gqa_bf16_matches_reference_fp32_kernel_config1():
    case = load_attn_case("config1")
    q, k, v, meta = _inputs(case)
    out = jb.packed_tree_attention_gqa(q, k, v, meta, case.scale, case.groups)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16
    assert_bf16_close(out, case.ref_out)
    assert jb.read_device_errors() == 0


def test_fp32_probability_fp32_output_within_reference_bound_config1():
    case = load_attn_case("config1")
    q, k, v, meta = _inputs(case)
    out = jb.packed_tree_attention_gqa(q, k, v, meta, case.scale, case.groups,
                                       output_dtype=torch.float32, fp32_probability=True)
    ref = paged_backend.packed_tree_attention(q, k, v, meta, case.scale, case.groups,
                                              backend="reference", output_dtype=torch.float32)
    torch.cuda.synchronize()
    for got in (out, ref):
        diff = (got.cpu() - case.ref_out).abs().max().item()
        assert diff <= FP32_BOUND, f"max-abs {diff:.3e} vs the reference fp32 kernel"
    rows = torch.from_numpy(case.fp64_rows)
    np.testing.assert_allclose(out.cpu()[rows].double().numpy(), case.fp64_out, rtol=0,
                               atol=FP32_BOUND)


def test_store_kernel_matches_reference_store_kvcache():
    z = load_npz("kv_store.npz")
    k = torch.from_numpy(z["k_before"]).to(DEV)
    v = torch.from_numpy(z["v_before"]).to(DEV)
    store_kvcache(torch.from_numpy(z["key"]).to(DEV), torch.from_numpy(z["value"]).to(DEV), k, v,
                  torch.from_numpy(z["slots"]).to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(k.cpu().numpy().view(np.uint32), z["k_after"].view(np.uint32))
    assert np.array_equal(v.cpu().numpy().view(np.uint32), z["v_after"].view(np.uint32))


def test_commit_kernel_matches_reference_copy_accepted_kv():
    z = load_npz("kv_commit.npz")
    pool = torch.from_numpy(z["before"]).to(DEV)
    nbytes = copy_accepted_kv(pool, torch.from_numpy(z["src"]).to(DEV),
                              torch.from_numpy(z["dst"]).to(DEV), 16)
    torch.cuda.synchronize()
    assert nbytes == int(z["nbytes"])
    assert np.array_equal(pool.cpu().numpy().view(np.uint32), z["after"].view(np.uint32))
