"""GPU parity of the sm_100a tree-attention kernel against the CPU oracle.

Cases follow the reference's qualification and sanity checks: the page/tile boundary
prefix sweep, NaN-poisoned unleased pages, request and off-branch isolation, the GQA
head mapping, strided operands, CUDA-graph replay with changed ragged metadata, plus
the benchmark configurations.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import tree_gqa, workloads
from oracle import tree_attention as attn_oracle

from helpers import (PREFIX_LENGTHS, assert_bf16_close, assert_fp32_close, bits_equal,
                     oracle_output, ragged_batch, run_gqa)

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)


def tensors(batch, dtype=torch.bfloat16, **kw):
    return workloads.make_tensors(batch, DEVICE, dtype, **kw)


def test_config1_matches_oracle_and_reference_fixture_shape():
    batch = workloads.config1()
    q, k, v = tensors(batch)
    out = run_gqa(batch, q, k, v)
    assert out.shape == (16, 32, 128) and out.dtype == torch.bfloat16
    assert_bf16_close(out, oracle_output(batch, q, k, v))
    assert jb.read_device_errors() == 0


@pytest.mark.parametrize("prefix", PREFIX_LENGTHS)
def test_page_and_tile_boundary_sweep(prefix):
    batch = ragged_batch((prefix, max(0, prefix - 1), prefix // 2))
    q, k, v = tensors(batch)
    expected = oracle_output(batch, q, k, v)
    assert_bf16_close(run_gqa(batch, q, k, v), expected)
    fp32 = run_gqa(batch, q, k, v, output_dtype=torch.float32, fp32_probability=True)
    assert fp32.dtype == torch.float32
    assert_fp32_close(fp32, expected)


@pytest.mark.parametrize("prefix", (0, 65, 257, 2048))
def test_fp32_output_round_trip_reproduces_bf16_store(prefix):
    batch = ragged_batch((prefix, 3, prefix + 1))
    q, k, v = tensors(batch)
    bf16 = run_gqa(batch, q, k, v)
    fp32 = run_gqa(batch, q, k, v, output_dtype=torch.float32)
    assert bits_equal(fp32.to(torch.bfloat16), bf16)


def test_reference_backends_use_fp32_probabilities():
    batch = ragged_batch((1024, 0, 257))
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    expected = oracle_output(batch, q, k, v)
    for backend in ("auto", "reference", "prefix"):
        out = jb.packed_tree_attention(q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                       backend=backend, output_dtype=torch.float32)
        assert_fp32_close(out, expected)
    gqa = jb.packed_tree_attention(q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                   backend="gqa")
    assert_bf16_close(gqa, expected)


@pytest.mark.parametrize("prefix", (0, 1, 63, 65, 256, 257, 2048))
def test_tcgen05_and_portable_cores_agree(prefix):
    batch = ragged_batch((prefix, max(0, prefix - 1), prefix // 2, prefix + 5),
                         counts=(63, 31, 47, 128))
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    outs = []
    for portable in (False, True):
        out = torch.empty(q.shape, dtype=torch.float32, device=DEVICE)
        tree_gqa.launch_tree_attention(out, q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                       portable_core=portable)
        outs.append(out)
    expected = oracle_output(batch, q, k, v)
    assert_bf16_close(outs[0], expected)
    assert_bf16_close(outs[1], expected)
    assert (outs[0] - outs[1]).abs().max().item() < 2e-3
    assert jb.read_device_errors() == 0


@pytest.mark.parametrize("split_keys", (1024, 2048))
def test_split_kv_partials_match_single_pass(split_keys):
    batch = ragged_batch((4096, 1500, 7000), counts=(64, 17, 128), kv_heads=2)
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    whole = torch.empty(q.shape, dtype=torch.float32, device=DEVICE)
    tree_gqa.launch_tree_attention(whole, q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                   split_keys=1 << 20)
    split = torch.empty_like(whole)
    tree_gqa.launch_tree_attention(split, q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                   split_keys=split_keys)
    portable = torch.empty_like(whole)
    tree_gqa.launch_tree_attention(portable, q, k, v, meta, batch.head_dim ** -0.5, batch.groups,
                                   split_keys=split_keys, portable_core=True)
    expected = oracle_output(batch, q, k, v)
    assert_bf16_close(whole, expected)
    assert_bf16_close(split, expected)
    assert_bf16_close(portable, expected)
    assert (whole - split).abs().max().item() < 1e-3


@pytest.mark.parametrize("prefix,nodes", ((512, 16), (512, 33), (512, 64), (1024, 16), (2048, 32),
                                          (500, 16), (0, 128), (4096, 128)))
def test_constant_values_give_exact_normalisation(prefix, nodes):
    # Every output row is a convex combination of V rows: with V constant the output is
    # that constant, whatever the scores.  Tile-aligned prefixes make every prefix tile a
    # TMA tile followed by a cp.async tree tile, the pattern that exposed a stage-reuse race.
    rng = np.random.default_rng(5)
    batch = workloads.build_batch([prefix], [workloads.random_parents(rng, nodes)], seed=11)
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    v_const = torch.full_like(v, 0.25)
    for _ in range(3):
        out = torch.empty(q.shape, dtype=torch.float32, device=DEVICE)
        tree_gqa.launch_tree_attention(out, q, k, v_const, meta, batch.head_dim ** -0.5,
                                       batch.groups)
        assert (out - 0.25).abs().max().item() < 1e-3
    assert jb.read_device_errors() == 0


def test_repeat_is_bitwise_deterministic():
    batch = ragged_batch((2048, 65, 0))
    q, k, v = tensors(batch)
    a = run_gqa(batch, q, k, v)
    b = run_gqa(batch, q, k, v)
    assert bits_equal(a, b)


def test_other_requests_cannot_affect_neighbors():
    batch = ragged_batch((65, 0, 257))
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    original = run_gqa(batch, q, k, v, meta)
    q2, k2, v2 = q.clone(), k.clone(), v.clone()
    q2[meta.request_slice(0)] *= 7
    slots = attn_oracle.request_slots(65, batch.block_tables[0], batch.tree_slots[0], 256).to(DEVICE)
    k2[slots // 256, slots % 256] *= -17
    v2[slots // 256, slots % 256] += 53
    changed = run_gqa(batch, q2, k2, v2, meta)
    for r in (1, 2):
        assert bits_equal(changed[meta.request_slice(r)], original[meta.request_slice(r)])
    assert not bits_equal(changed[meta.request_slice(0)], original[meta.request_slice(0)])


def test_off_branch_kv_cannot_affect_ancestor_path():
    batch = ragged_batch((65, 0, 257))
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    original = run_gqa(batch, q, k, v, meta)
    parents = batch.parents[0]
    chosen = len(parents) - 1
    path = attn_oracle.parent_chain(parents, chosen)
    off = [n for n in range(len(parents)) if n not in path]
    slots = torch.tensor([batch.tree_slots[0][n] for n in off], device=DEVICE)
    k2, v2 = k.clone(), v.clone()
    k2[slots // 256, slots % 256] *= 97
    v2[slots // 256, slots % 256] += 113
    changed = run_gqa(batch, q, k2, v2, meta)
    assert bits_equal(changed[path], original[path])


def test_kv_head_maps_only_to_its_query_heads():
    batch = ragged_batch((0, 255, 257), kv_heads=8)
    q, k, v = tensors(batch)
    base = run_gqa(batch, q, k, v)
    v2 = v.clone()
    v2[:, :, 2] += 3
    poisoned = run_gqa(batch, q, k, v2)
    assert bits_equal(base[:, :8], poisoned[:, :8])
    assert bits_equal(base[:, 12:], poisoned[:, 12:])
    assert not torch.equal(base[:, 8:12], poisoned[:, 8:12])


@pytest.mark.parametrize("groups,head_dim", ((1, 64), (4, 128), (8, 128), (16, 64), (2, 128)))
def test_strided_operands_and_gqa_geometry(groups, head_dim):
    batch = ragged_batch((63, 64, 65), kv_heads=2, groups=groups, head_dim=head_dim)
    q, k, v = tensors(batch)
    expected = oracle_output(batch, q, k, v)
    qs = torch.empty((q.shape[0] * 2, q.shape[1] * 2, head_dim), dtype=q.dtype, device=DEVICE)[::2, ::2]
    qs.copy_(q)
    pools = []
    for pool in (k, v):
        wide = torch.empty((pool.shape[0] * 2, pool.shape[1], pool.shape[2] * 2, head_dim),
                           dtype=pool.dtype, device=DEVICE)[::2, :, ::2]
        wide.copy_(pool)
        pools.append(wide)
    out = run_gqa(batch, qs, pools[0], pools[1])
    assert_bf16_close(out, expected)


def test_fp16_operands():
    batch = ragged_batch((257, 1, 1024))
    q, k, v = tensors(batch, dtype=torch.float16)
    assert_bf16_close(run_gqa(batch, q, k, v), oracle_output(batch, q, k, v))


def test_cuda_graph_replay_follows_changed_ragged_metadata():
    first = ragged_batch((0, 255, 256, 257), counts=(63, 31, 47, 63), seed=91, num_blocks=16)
    q, k, v = tensors(first)
    meta = first.metadata(DEVICE)
    run_gqa(first, q, k, v, meta)  # warm-up outside capture
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        result = run_gqa(first, q, k, v, meta)
    # Same Q, R and sum(T^2) with different prefixes, node counts and slots.
    second = ragged_batch((257, 0, 255, 256), counts=(31, 63, 63, 47), seed=92, num_blocks=16)
    assert second.total_queries == first.total_queries
    other = second.metadata(DEVICE)
    assert other.qq_bias.numel() == meta.qq_bias.numel()
    q2, k2, v2 = tensors(second)
    for field in ("cu_seqlens_q", "query_to_request", "query_local_row", "prefix_lens",
                  "node_counts", "tree_slots", "qq_bias", "qq_bias_offsets"):
        getattr(meta, field).copy_(getattr(other, field))
    meta.block_tables.fill_(-1)
    meta.block_tables[:, :other.block_tables.shape[1]].copy_(other.block_tables)
    q.copy_(q2)
    k.copy_(k2)
    v.copy_(v2)
    graph.replay()
    torch.cuda.synchronize()
    fresh = run_gqa(second, q, k, v, other)
    assert bits_equal(result, fresh)
    assert_bf16_close(result, oracle_output(second, q, k, v))


def test_config2_matches_oracle():
    batch = workloads.config2()
    q, k, v = tensors(batch)
    assert_bf16_close(run_gqa(batch, q, k, v), oracle_output(batch, q, k, v))


def test_config3_serving_mix_matches_oracle():
    batch = workloads.config3()
    q, k, v = workloads.make_tensors(batch, DEVICE, generator_device="cuda")
    out = run_gqa(batch, q, k, v)
    # Every request is checked; the oracle runs on CPU request by request.
    assert_bf16_close(out, oracle_output(batch, q, k, v))


def test_config4_long_context_sample_and_full_size_property():
    batch = workloads.config4()
    q, k, v = workloads.make_tensors(batch, DEVICE, generator_device="cuda")
    out = run_gqa(batch, q, k, v)
    rows = slice(0, batch.node_counts[0] + batch.node_counts[1])
    assert_bf16_close(out, oracle_output(batch, q, k, v, requests=(0, 1)), rows=rows)
    # Size-independent property at full size: a constant V makes every output row that
    # constant (probabilities sum to one over every visible key of every request).
    live = torch.from_numpy(batch.live_slots()).to(DEVICE)
    v_const = torch.full_like(v, float("nan"))
    v_const.view(-1, batch.num_kv_heads, batch.head_dim)[live] = 0.375
    const = run_gqa(batch, q, k, v_const, output_dtype=torch.float32)
    assert (const - 0.375).abs().max().item() < 1e-3


def test_invalid_arguments_raise_before_launch():
    batch = ragged_batch((65,), counts=(5,))
    q, k, v = tensors(batch)
    meta = batch.metadata(DEVICE)
    with pytest.raises(ValueError, match="query tile"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, batch.groups, query_tile=2)
    with pytest.raises(ValueError, match="BF16 or FP16"):
        jb.packed_tree_attention_gqa(q.float(), k, v, meta, 0.1, batch.groups)
    with pytest.raises(ValueError, match="GQA"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, 3)
    with pytest.raises(ValueError, match="grouping"):
        jb.packed_tree_attention_gqa(q, k, v, meta, 0.1, 2)
    with pytest.raises(ValueError, match="metadata"):
        jb.packed_tree_attention_gqa(q[:-1], k, v, meta, 0.1, batch.groups)
    with pytest.raises(ValueError, match="backend"):
        jb.packed_tree_attention(q, k, v, meta, 0.1, batch.groups, backend="triton")
