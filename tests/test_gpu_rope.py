"""Fused HF-order RoPE + node K/V scatter kernel: bit-exact against the reference's golden
output and the eager oracle (tree_fusion.py byte-exact gates, tests/test_jetspec_tree_fusion.py)."""
from __future__ import annotations

import pytest
import torch

import jetspec_b200 as jb
from golden_cases import load_rope_case
from oracle import rope as rope_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def bits_equal(a, b):
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(
        a.contiguous().view(torch.uint8).cpu(), b.contiguous().view(torch.uint8).cpu())


@pytest.mark.parametrize("dtype_name", ["bf16", "f32"])
def test_matches_reference_golden(dtype_name):
    q, k, v, positions, cache, slots, out_ref, kv_ref = load_rope_case(dtype_name, DEV)
    gen = torch.Generator(device=DEV).manual_seed(3)
    pools = torch.randn((2, 4, 256) + tuple(k.shape[1:]), generator=gen, device=DEV).to(k.dtype)
    before = pools.clone()
    out = jb.rope_scatter(q, k, v, positions, cache, pools[0], pools[1], slots)
    torch.cuda.synchronize()
    assert bits_equal(out, out_ref)
    assert bits_equal(pools[:, slots // 256, slots % 256], kv_ref)
    before[:, slots // 256, slots % 256] = pools[:, slots // 256, slots % 256]
    assert bits_equal(pools, before), "a row outside the node slots was written"
    assert jb.read_device_errors() == 0


def _case(dtype, *, strided, cache_rank, rows=300, q_heads=32, kv_heads=8, dim=128,
          index_dtype=torch.int64, cache_dtype=torch.float32):
    gen = torch.Generator(device=DEV).manual_seed(11)

    def values(heads):
        if strided:
            backing = torch.randn(rows * 2, heads * 2, dim * 2, generator=gen, device=DEV).to(dtype)
            return backing[::2, ::2, ::2]
        return torch.randn(rows, heads, dim, generator=gen, device=DEV).to(dtype)

    q, k, v = values(q_heads), values(kv_heads), values(kv_heads)
    positions = torch.randint(0, 4096, (rows,), generator=gen, device=DEV).to(index_dtype)
    slots = torch.randperm(8 * 256, generator=gen, device=DEV)[:rows].to(index_dtype)
    angles = torch.arange(4096, device=DEV, dtype=torch.float32)[:, None] * (
        torch.arange(dim // 2, device=DEV, dtype=torch.float32)[None, :] + 1) * .00317
    cache = torch.cat((angles.cos(), angles.sin()), -1).to(cache_dtype)
    if cache_rank == 3:
        cache = cache.unsqueeze(1)
    pools = torch.randn(2, 8, 256, kv_heads, dim, generator=gen, device=DEV).to(dtype)
    return q, k, v, positions, cache, pools, slots


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("strided", [False, True])
@pytest.mark.parametrize("cache_rank", [2, 3])
def test_matches_eager_oracle(dtype, strided, cache_rank):
    q, k, v, positions, cache, pools, slots = _case(dtype, strided=strided, cache_rank=cache_rank)
    ref_pools = pools.cpu()
    expected = rope_oracle.rope_scatter(q, k, v, positions, cache, ref_pools[0], ref_pools[1], slots)
    out = jb.rope_scatter_prevalidated(q, k, v, positions, cache, pools[0], pools[1], slots,
                                       torch.empty_like(q))
    torch.cuda.synchronize()
    assert bits_equal(out, expected)
    assert bits_equal(pools, ref_pools)


def test_int32_indices_bf16_cache():
    q, k, v, positions, cache, pools, slots = _case(torch.bfloat16, strided=False, cache_rank=2,
                                                    index_dtype=torch.int32,
                                                    cache_dtype=torch.bfloat16)
    ref_pools = pools.cpu()
    expected = rope_oracle.rope_scatter(q, k, v, positions, cache, ref_pools[0], ref_pools[1], slots)
    out = jb.rope_scatter(q, k, v, positions, cache, pools[0], pools[1], slots)
    torch.cuda.synchronize()
    assert bits_equal(out, expected) and bits_equal(pools, ref_pools)


def test_device_value_checks_of_the_external_boundary():
    q, k, v, positions, cache, pools, slots = _case(torch.bfloat16, strided=False, cache_rank=2,
                                                    rows=16)
    with pytest.raises(ValueError, match="positions lie outside"):
        bad = positions.clone()
        bad[3] = 5000
        jb.rope_scatter(q, k, v, bad, cache, pools[0], pools[1], slots)
    with pytest.raises(ValueError, match="slots lie outside"):
        bad = slots.clone()
        bad[0] = 8 * 256
        jb.rope_scatter(q, k, v, positions, cache, pools[0], pools[1], bad)
    with pytest.raises(ValueError, match="unique"):
        bad = slots.clone()
        bad[1] = bad[0]
        jb.rope_scatter(q, k, v, positions, cache, pools[0], pools[1], bad)
    with pytest.raises(ValueError, match="alias"):
        jb.rope_scatter(q, k, v, positions, cache, pools[0], pools[1], slots, out=q)
