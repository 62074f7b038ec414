"""fp32 q / k / v through the dispatcher's auto / reference / prefix backends.

The reference runs those backends on fp32 operands as well as bf16 / f16
(nanovllm/speculative/jetspec/paged_backend.py:240-306, tree_attention.py:21-62), and its
own qualification runs c1 / c2 / c3 in both dtypes and asserts that the packed launch is
byte-equal to independent per-request launches (tests/test_jetspec_packed_attention.py:
156-171).  Here fp32 operands run on the CUDA-core fp32 kernel; results are held to the
fp32 masked-SDPA oracle within the reference's fp32 bound (1e-4 scaled max-abs and
relative RMS, benchmarks/jetspec_numeric_oracles.py:21) and to the reference kernel's own
golden output.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import workloads

from golden_cases import load_attn_case
from helpers import FP32_BOUND, assert_bf16_close, assert_fp32_close, bits_equal, oracle_output, ragged_batch

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)
BACKENDS = ("auto", "reference", "prefix")


def _tensors(batch, dtype, poison=True):
    return workloads.make_tensors(batch, DEVICE, dtype=dtype, poison=poison)


@pytest.mark.parametrize("counts", ((63,), (63, 31), (63, 31, 47)))
@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
def test_c1_c2_c3_in_both_dtypes_against_the_oracle(counts, dtype):
    prefixes = (65, 0, 257)[:len(counts)]
    batch = ragged_batch(prefixes, counts=counts)
    q, k, v = _tensors(batch, dtype)
    meta = batch.metadata(DEVICE)
    expected = oracle_output(batch, q, k, v)
    for backend in BACKENDS:
        out = jb.packed_tree_attention(q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                       backend=backend, output_dtype=torch.float32)
        assert out.dtype == torch.float32
        assert_fp32_close(out, expected)
    native = jb.packed_tree_attention(q, k, v, meta, batch.head_dim ** -0.5, batch.groups)
    assert native.dtype == dtype
    if dtype == torch.float32:
        assert_fp32_close(native, expected)
    else:
        assert_bf16_close(native, expected)
    assert jb.read_device_errors() == 0


def test_fp32_packed_launch_is_byte_equal_to_per_request_launches():
    """The reference's c1..c3 property: packing requests changes no output byte."""
    counts = (63, 31, 47)
    batch = ragged_batch((65, 0, 257), counts=counts)
    q, k, v = _tensors(batch, torch.float32)
    scale = batch.head_dim ** -0.5
    packed = jb.packed_tree_attention(q, k, v, batch.metadata(DEVICE), scale, batch.groups)
    offsets = np.concatenate(([0], np.cumsum(counts)))
    for r in range(len(counts)):
        single = workloads.TreeBatch([batch.prefix_lens[r]], [batch.parents[r]],
                                     [batch.block_tables[r]], [batch.owned_pages[r]],
                                     [batch.tree_slots[r]], [batch.accepted_paths[r]],
                                     batch.num_blocks, num_kv_heads=batch.num_kv_heads,
                                     groups=batch.groups, head_dim=batch.head_dim)
        rows = slice(int(offsets[r]), int(offsets[r + 1]))
        alone = jb.packed_tree_attention(q[rows].contiguous(), k, v, single.metadata(DEVICE),
                                         scale, batch.groups)
        assert bits_equal(alone, packed[rows])


def test_fp32_operands_match_the_reference_fp32_kernel_golden():
    """Golden config 1: the reference's _packed_paged_tree_fp32 output on these operands
    (bf16 values, which fp32 holds exactly) and its fp64 parent-chain rows."""
    case = load_attn_case("config1")
    from jetspec_b200.packed_metadata import PackedTreeMetadata

    meta = PackedTreeMetadata.from_parents(case.prefixes, case.tables, case.parents,
                                           case.tree_slots, 256, device=DEVICE)
    q = case.q.to(DEVICE).float()
    k, v = case.k_pool.to(DEVICE).float(), case.v_pool.to(DEVICE).float()
    for backend in BACKENDS:
        out = jb.packed_tree_attention(q, k, v, meta, case.scale, case.groups, backend=backend)
        diff = (out.cpu() - case.ref_out).abs().max().item()
        assert diff <= FP32_BOUND, f"{backend}: max-abs {diff:.3e} vs the reference fp32 kernel"
        rows = torch.from_numpy(case.fp64_rows)
        np.testing.assert_allclose(out.cpu()[rows].double().numpy(), case.fp64_out, rtol=0,
                                   atol=FP32_BOUND)


@pytest.mark.parametrize("groups,head_dim", ((1, 128), (8, 128), (16, 64), (4, 64)))
def test_fp32_group_and_head_dim_variants(groups, head_dim):
    batch = ragged_batch((300, 1, 1024), counts=(17, 64, 5), kv_heads=2, groups=groups,
                         head_dim=head_dim)
    q, k, v = _tensors(batch, torch.float32)
    out = jb.packed_tree_attention(q, k, v, batch.metadata(DEVICE), head_dim ** -0.5, groups,
                                   backend="reference")
    assert_fp32_close(out, oracle_output(batch, q, k, v))


def test_fp32_strided_pools_and_isolation():
    """K/V pools as views of the reference's [2, layers, blocks, bs, heads, dim] pool (layer
    1 of 2), and perturbing one request's prefix, nodes and queries leaves every other
    request's bytes unchanged."""
    batch = ragged_batch((65, 0, 257), counts=(63, 31, 47))
    q, k, v = _tensors(batch, torch.float32, poison=False)
    pool = torch.zeros((2, 2) + tuple(k.shape), dtype=torch.float32, device=DEVICE)
    pool[0, 1].copy_(k)
    pool[1, 1].copy_(v)
    kp, vp = pool[0, 1], pool[1, 1]
    meta = batch.metadata(DEVICE)
    scale = batch.head_dim ** -0.5
    base = jb.packed_tree_attention(q, kp, vp, meta, scale, batch.groups)
    assert_fp32_close(base, oracle_output(batch, q, k, v))
    q2 = q.clone()
    q2[:63] *= 31
    slots = torch.tensor(batch.tree_slots[0], device=DEVICE)
    kp[slots // 256, slots % 256] *= -17
    vp[slots // 256, slots % 256] += 53
    changed = jb.packed_tree_attention(q2, kp, vp, meta, scale, batch.groups)
    assert bits_equal(changed[63:], base[63:])
    assert not torch.equal(changed[:63], base[:63])


def test_fp32_graph_replay_with_restaged_metadata():
    """Capture once, restage the trees' ancestor bias in place (same node counts, new
    random parents), replay: the replay must see the new trees."""
    from jetspec_b200.packed_metadata import PackedTreeMetadata

    batch = ragged_batch((65, 0, 257), counts=(63, 31, 47))
    q, k, v = _tensors(batch, torch.float32)
    meta = batch.metadata(DEVICE)
    scale = batch.head_dim ** -0.5
    holder = {}
    jb.packed_tree_attention(q, k, v, meta, scale, batch.groups)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        holder["out"] = jb.packed_tree_attention(q, k, v, meta, scale, batch.groups)
    rng = np.random.default_rng(99)
    parents = [workloads.random_parents(rng, len(p)) for p in batch.parents]
    restaged = PackedTreeMetadata.from_parents(batch.prefix_lens, batch.block_tables, parents,
                                               batch.tree_slots, 256, device=DEVICE)
    meta.qq_bias.copy_(restaged.qq_bias)
    graph.replay()
    torch.cuda.synchronize()
    other = workloads.TreeBatch(batch.prefix_lens, parents, batch.block_tables,
                                batch.owned_pages, batch.tree_slots, batch.accepted_paths,
                                batch.num_blocks, num_kv_heads=batch.num_kv_heads,
                                groups=batch.groups, head_dim=batch.head_dim)
    assert_fp32_close(holder["out"], oracle_output(other, q, k, v))


def test_gqa_backend_keeps_rejecting_fp32_like_the_reference():
    batch = ragged_batch((65,), counts=(16,))
    q, k, v = _tensors(batch, torch.float32)
    with pytest.raises(ValueError, match="BF16 or FP16"):
        jb.packed_tree_attention(q, k, v, batch.metadata(DEVICE), 0.1, batch.groups,
                                 backend="gqa")
