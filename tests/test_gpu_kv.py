"""GPU bit-exactness of the paged KV store, tree-node scatter and accepted-only commit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import workloads
from oracle import kv_cache as kv_oracle

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)


def raw(t: torch.Tensor) -> np.ndarray:
    view = {2: torch.int16, 4: torch.int32}[t.element_size()]
    return t.detach().cpu().contiguous().view(view).numpy().copy()


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
@pytest.mark.parametrize("slot_dtype", (torch.int32, torch.int64))
def test_store_kvcache_bit_exact_with_padding_slots(dtype, slot_dtype):
    gen = torch.Generator().manual_seed(5)
    blocks, bs, heads, dim, n = 6, 256, 8, 128, 300
    key = torch.randn((n, heads, dim), generator=gen).to(dtype)
    value = torch.randn((n, heads, dim), generator=gen).to(dtype)
    slots = torch.randperm(blocks * bs, generator=gen)[:n]
    slots[::7] = -1
    k_cache = torch.randn((blocks, bs, heads, dim), generator=gen).to(dtype)
    v_cache = torch.randn((blocks, bs, heads, dim), generator=gen).to(dtype)
    ek, ev = raw(k_cache), raw(v_cache)
    kv_oracle.store_kvcache(raw(key), raw(value), ek, ev, slots.numpy())
    kc, vc = k_cache.to(DEVICE), v_cache.to(DEVICE)
    jb.store_kvcache(key.to(DEVICE), value.to(DEVICE), kc, vc, slots.to(DEVICE, slot_dtype))
    assert np.array_equal(raw(kc), ek) and np.array_equal(raw(vc), ev)


def test_store_kvcache_keeps_reference_assertions():
    key = torch.zeros((4, 2, 128), dtype=torch.bfloat16, device=DEVICE)
    cache = torch.zeros((1, 256, 2, 128), dtype=torch.bfloat16, device=DEVICE)
    slots = torch.arange(4, device=DEVICE)
    with pytest.raises(AssertionError):
        jb.store_kvcache(key.transpose(1, 2).contiguous().transpose(1, 2), key, cache, cache, slots)
    with pytest.raises(AssertionError):
        jb.store_kvcache(key, key, cache, cache, slots[:3])


def test_scatter_tree_kv_strided_rows_bit_exact():
    batch = workloads.config1()
    meta = batch.metadata(DEVICE)
    gen = torch.Generator().manual_seed(9)
    wide_k = torch.randn((16, 16, 128), generator=gen).bfloat16()
    wide_v = torch.randn((16, 16, 128), generator=gen).bfloat16()
    k_rows, v_rows = wide_k[:, ::2], wide_v[:, ::2]  # [16, 8, 128] with head stride 256
    k_pool = torch.full((5, 256, 8, 128), float("nan"), dtype=torch.bfloat16)
    v_pool = k_pool.clone()
    ek, ev = raw(k_pool), raw(v_pool)
    slots = np.asarray(batch.tree_slots[0])
    ek.reshape(-1, 8, 128)[slots] = raw(k_rows)
    ev.reshape(-1, 8, 128)[slots] = raw(v_rows)
    kp, vp = k_pool.to(DEVICE), v_pool.to(DEVICE)
    jb.scatter_tree_kv(k_rows.to(DEVICE), v_rows.to(DEVICE), kp, vp, meta.tree_slots)
    assert np.array_equal(raw(kp), ek) and np.array_equal(raw(vp), ev)


def _pool(layers, blocks, heads=2, dim=128, dtype=torch.bfloat16, seed=11):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn((2, layers, blocks, 256, heads, dim), generator=gen).to(dtype)


@pytest.mark.parametrize("slot_dtype", (torch.int32, torch.int64))
def test_commit_bit_exact_all_layers(slot_dtype):
    pool = _pool(3, 8)
    src = [6 * 256 + i for i in (0, 1, 8, 15, 40)]
    dst = [2 * 256 + 10 + i for i in range(5)]
    expected = raw(pool)
    payload = kv_oracle.copy_accepted_kv(expected, np.asarray(src), np.asarray(dst), 256)
    device_pool = pool.to(DEVICE)
    got = jb.copy_accepted_kv(device_pool, torch.tensor(src, dtype=slot_dtype, device=DEVICE),
                              torch.tensor(dst, dtype=slot_dtype, device=DEVICE), 256)
    assert got == payload == 5 * 2 * 3 * 2 * 128 * 2
    assert np.array_equal(raw(device_pool), expected)


def test_commit_overlapping_sources_and_destinations():
    pool = _pool(2, 4)
    # A chain of moves where destinations are also later sources: the reference
    # materialises the gather first, so every destination gets the ORIGINAL source row.
    src = [10, 11, 12, 13, 300]
    dst = [11, 12, 13, 14, 10]
    expected = raw(pool)
    kv_oracle.copy_accepted_kv(expected, np.asarray(src), np.asarray(dst), 256)
    device_pool = pool.to(DEVICE)
    jb.copy_accepted_kv(device_pool, torch.tensor(src, device=DEVICE),
                        torch.tensor(dst, device=DEVICE), 256)
    assert np.array_equal(raw(device_pool), expected)


def test_commit_qwen3_geometry_36_layers():
    gen = torch.Generator().manual_seed(3)
    pool = torch.randn((2, 36, 12, 256, 8, 128), generator=gen).bfloat16()
    perm = torch.randperm(12 * 256, generator=gen)
    src, dst = perm[:250], perm[250:500]
    expected = raw(pool)
    kv_oracle.copy_accepted_kv(expected, src.numpy(), dst.numpy(), 256)
    device_pool = pool.to(DEVICE)
    got = jb.copy_accepted_kv(device_pool, src.to(DEVICE), dst.to(DEVICE), 256)
    assert got == 250 * 2 * 36 * 8 * 128 * 2
    assert np.array_equal(raw(device_pool), expected)


def test_commit_config3_paths_and_empty_commit():
    batch = workloads.config3()
    src, dst = batch.commit_slots()
    gen = torch.Generator().manual_seed(4)
    # A compact pool holding just the touched pages keeps this test small.
    pages = sorted({s // 256 for s in src + dst})
    remap = {p: i for i, p in enumerate(pages)}
    src_c = [remap[s // 256] * 256 + s % 256 for s in src]
    dst_c = [remap[s // 256] * 256 + s % 256 for s in dst]
    pool = torch.randn((2, 1, len(pages), 256, 8, 128), generator=gen).bfloat16()
    expected = raw(pool)
    kv_oracle.copy_accepted_kv(expected, np.asarray(src_c), np.asarray(dst_c), 256)
    device_pool = pool.to(DEVICE)
    jb.copy_accepted_kv(device_pool, torch.tensor(src_c, device=DEVICE),
                        torch.tensor(dst_c, device=DEVICE), 256)
    assert np.array_equal(raw(device_pool), expected)
    empty = torch.empty(0, dtype=torch.int64, device=DEVICE)
    assert jb.copy_accepted_kv(device_pool, empty, empty, 256) == 0


@pytest.mark.parametrize("layers,heads,dim,n", [(1, 1, 64, 300), (1, 1, 128, 13000)])
def test_commit_grid_wide_form_bit_exact(layers, heads, dim, n):
    """Commits the plane-local form does not take: too few planes (one layer, one head,
    64-dim rows: 16 one-word planes) and more slots than one CTA's staging holds (13 000);
    both go through the cooperative grid-wide kernel.  Sources and destinations overlap
    (a shifted chain), so the grid barrier between gather and scatter is exercised."""
    gen = torch.Generator().manual_seed(21)
    blocks = (2 * n) // 256 + 2
    pool = torch.randn((2, layers, blocks, 256, heads, dim), generator=gen).bfloat16()
    perm = torch.randperm(blocks * 256, generator=gen)
    src = perm[:n]
    dst = perm[n // 2:n // 2 + n]  # half of the destinations are also sources
    expected = raw(pool)
    kv_oracle.copy_accepted_kv(expected, src.numpy(), dst.numpy(), 256)
    device_pool = pool.to(DEVICE)
    jb.copy_accepted_kv(device_pool, src.to(DEVICE), dst.to(DEVICE), 256)
    assert np.array_equal(raw(device_pool), expected)


def test_commit_rejects_bad_slot_maps():
    pool = _pool(1, 2).to(DEVICE)
    with pytest.raises(ValueError, match="one-dimensional"):
        jb.copy_accepted_kv(pool, torch.zeros((2, 2), dtype=torch.long, device=DEVICE),
                            torch.zeros(4, dtype=torch.long, device=DEVICE), 256)
    with pytest.raises(ValueError, match="differ"):
        jb.copy_accepted_kv(pool, torch.zeros(3, dtype=torch.long, device=DEVICE),
                            torch.zeros(4, dtype=torch.long, device=DEVICE), 256)
    assert jb.read_device_errors() == 0
