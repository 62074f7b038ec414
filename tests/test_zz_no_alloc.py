"""The allocation-free tree-attention entry point against the workspace entry point.

jt_tree_attn_launch_noalloc exists for callers that cannot allocate device memory, such
as a host that binds only the C ABI and keeps every device byte in its own fixed arenas:
it takes its scratch from a static device array inside the library.  This test calls it
through the C ABI with no workspace and checks two calls in a row against
jt_tree_attn_launch on the same inputs and against the fp32 masked-SDPA oracle, on the
portable core as well as the tcgen05 core, and on a geometry whose split-KV partial
results do not fit the static array's partial budget, so that its device plan takes
coarser splits than the workspace entry point's.  The file name makes pytest collect it
last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from jetspec_b200 import _launch, _lib, workloads

from helpers import BF16_MAX_ABS, BF16_MEAN_ABS, assert_bf16_close, oracle_output

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)


def _params(out, q, k, v, meta, groups, split_keys, flags=0):
    p = _lib.JtTreeAttnParams()
    p.out, p.q, p.k_pool, p.v_pool = out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.cu_seqlens_q = meta.cu_seqlens_q.data_ptr()
    p.query_to_request = meta.query_to_request.data_ptr()
    p.query_local_row = meta.query_local_row.data_ptr()
    p.prefix_lens = meta.prefix_lens.data_ptr()
    p.node_counts = meta.node_counts.data_ptr()
    p.block_tables = meta.block_tables.data_ptr()
    p.tree_slots = meta.tree_slots.data_ptr()
    p.qq_bias = meta.qq_bias.data_ptr()
    p.qq_bias_offsets = meta.qq_bias_offsets.data_ptr()
    p.num_requests, p.total_queries = meta.num_requests, meta.total_queries
    p.num_kv_heads, p.groups, p.head_dim = k.shape[2], groups, q.shape[2]
    p.block_size, p.table_width = meta.block_size, meta.block_tables.shape[1]
    p.dtype = p.out_dtype = _lib.JT_BF16
    p.flags = flags
    p.num_blocks = k.shape[0]
    p.q_stride0, p.q_stride1 = q.stride(0), q.stride(1)
    p.out_stride0, p.out_stride1 = out.stride(0), out.stride(1)
    p.table_stride0 = meta.block_tables.stride(0)
    p.k_stride0, p.k_stride1, p.k_stride2 = k.stride(0), k.stride(1), k.stride(2)
    p.v_stride0, p.v_stride1, p.v_stride2 = v.stride(0), v.stride(1), v.stride(2)
    p.scale = q.shape[2] ** -0.5
    p.split_keys = split_keys
    return p


def _with_workspace(lib, out, q, k, v, meta, groups, split_keys, flags=0):
    size = ctypes.c_size_t(0)
    _lib.check(lib.jt_tree_attn_workspace_size(meta.num_requests, meta.total_queries, k.shape[2],
                                               groups, q.shape[2], ctypes.byref(size)))
    scratch = torch.empty(size.value, dtype=torch.uint8, device=DEVICE)
    p = _params(out, q, k, v, meta, groups, split_keys, flags)
    p.workspace, p.workspace_bytes = scratch.data_ptr(), scratch.numel()
    _lib.check(lib.jt_tree_attn_launch(ctypes.byref(p), _launch.stream_handle(DEVICE)))
    torch.cuda.synchronize(DEVICE)


def _without_workspace(lib, out, q, k, v, meta, groups, split_keys, flags=0):
    p = _params(out, q, k, v, meta, groups, split_keys, flags)
    p.workspace, p.workspace_bytes = None, 0
    _lib.check(lib.jt_tree_attn_launch_noalloc(ctypes.byref(p), _launch.stream_handle(DEVICE)))
    torch.cuda.synchronize(DEVICE)


def test_noalloc_entry_matches_workspace_entry_on_two_calls():
    lib = _lib.load_library()
    batch = workloads.config2()
    meta = batch.metadata(DEVICE)
    q, k, v = workloads.make_tensors(batch, DEVICE)
    # First call: automatic split plan.  Second call: 1024-key splits, so the partial
    # results and split counters left in the static array by the first call are reused.
    for split_keys in (0, 1024):
        expected = torch.empty_like(q)
        _with_workspace(lib, expected, q, k, v, meta, batch.groups, split_keys)
        got = torch.full_like(q, float("nan"))
        _without_workspace(lib, got, q, k, v, meta, batch.groups, split_keys)
        assert torch.isfinite(got).all()
        diff = (got.float() - expected.float()).abs()
        assert diff.max().item() <= BF16_MAX_ABS, diff.max().item()
        assert diff.mean().item() <= BF16_MEAN_ABS, diff.mean().item()


def _close(got, expected):
    assert torch.isfinite(got).all()
    diff = (got.float() - expected.float()).abs()
    assert diff.max().item() <= BF16_MAX_ABS, diff.max().item()
    assert diff.mean().item() <= BF16_MEAN_ABS, diff.mean().item()


def test_noalloc_entry_matches_the_oracle_on_both_cores():
    """Two calls in a row per core (the second reuses what the first left in the static
    array), each held to the fp32 masked-SDPA oracle and to the workspace entry point."""
    lib = _lib.load_library()
    batch = workloads.config2()
    meta = batch.metadata(DEVICE)
    q, k, v = workloads.make_tensors(batch, DEVICE)
    expected_oracle = oracle_output(batch, q, k, v)
    for flags in (0, _lib.JT_FLAG_PORTABLE_CORE):
        expected = torch.empty_like(q)
        _with_workspace(lib, expected, q, k, v, meta, batch.groups, 0, flags)
        for _ in range(2):
            got = torch.full_like(q, float("nan"))
            _without_workspace(lib, got, q, k, v, meta, batch.groups, 0, flags)
            _close(got, expected)
            assert_bf16_close(got, expected_oracle)


def test_noalloc_plan_is_coarser_when_partials_exceed_the_static_budget():
    """Config 4 (16 requests x 32768-key prefixes, 64-node trees) with 1024-key splits
    requested.  The workspace entry point sizes its partials for 4 x 48 query tiles x 8
    KV heads = 1536 slots and settles on 8192-key splits; the static array's 16 MiB hold
    256 slots, too few for any split, so its plan runs every item unsplit.  Both must
    still match each other and the oracle (one sampled request)."""
    lib = _lib.load_library()
    batch = workloads.config4()
    meta = batch.metadata(DEVICE)
    q, k, v = workloads.make_tensors(batch, DEVICE, poison=False, generator_device="cuda")
    expected = torch.empty_like(q)
    _with_workspace(lib, expected, q, k, v, meta, batch.groups, 1024)
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        _without_workspace(lib, got, q, k, v, meta, batch.groups, 1024)
        _close(got, expected)
    rows = slice(0, 64)  # request 0
    ref = oracle_output(batch, q, k, v, requests=[0])
    assert_bf16_close(got[rows], ref[rows])
    assert_bf16_close(expected[rows], ref[rows])
