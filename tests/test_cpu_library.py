"""The C ABI library without a GPU: it loads, exports every header symbol, and rejects
bad arguments with the documented status codes before touching the device."""
from __future__ import annotations

import ctypes
from pathlib import Path
import re

import pytest

from jetspec_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "jetspec_b200.h"


def header_functions():
    text = HEADER.read_text()
    body = text[text.index('extern "C" {'):]
    return sorted(set(re.findall(r"^\s*(?:int|int32_t|const char\*)\s+(jt_[a-z0-9_]+)\s*\(",
                                 body, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load_library()


def test_header_declares_the_boundary():
    names = header_functions()
    assert {"jt_tree_attn_launch", "jt_tree_attn_workspace_size", "jt_kv_store_launch",
            "jt_kv_commit_launch", "jt_last_error", "jt_abi_version"} <= set(names)


def test_library_exports_every_header_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), f"libjetspec_b200.so lacks {name}"
    assert set(header_functions()) <= set(_lib.EXPORTED_SYMBOLS)


def test_abi_version_and_limits(lib):
    assert lib.jt_abi_version() == _lib.ABI_VERSION
    assert lib.jt_kv_commit_max_slots() > 0


def test_null_parameters_are_rejected(lib):
    assert lib.jt_tree_attn_launch(None, None) == _lib.JT_ERR_INVALID
    assert b"null" in lib.jt_last_error()
    assert lib.jt_tree_attn_launch_noalloc(None, None) == _lib.JT_ERR_INVALID
    assert lib.jt_kv_store_launch(None, None) == _lib.JT_ERR_INVALID
    assert lib.jt_kv_commit_launch(None, None) == _lib.JT_ERR_INVALID
    assert lib.jt_rope_scatter_launch(None, None) == _lib.JT_ERR_INVALID
    assert lib.jt_accept_walk_launch(None, None) == _lib.JT_ERR_INVALID
    assert lib.jt_metadata_build_launch(None, None) == _lib.JT_ERR_INVALID
    assert lib.jt_row_linear_launch(None, None) == _lib.JT_ERR_INVALID


def test_accept_and_metadata_geometry_checks_precede_the_device(lib):
    import ctypes

    walk = _lib.JtAcceptWalkParams()
    walk.num_requests, walk.vocab, walk.max_depth, walk.num_nodes = 2, 100, 4, 10
    walk.path_stride, walk.logits_stride0 = 4, 100  # path_stride < max_depth + 1
    assert lib.jt_accept_walk_launch(ctypes.byref(walk), None) == _lib.JT_ERR_INVALID
    assert b"geometry" in lib.jt_last_error()
    walk.path_stride = 5  # geometry valid, tensors missing
    assert lib.jt_accept_walk_launch(ctypes.byref(walk), None) == _lib.JT_ERR_INVALID
    assert b"null" in lib.jt_last_error()
    meta = _lib.JtMetadataBuildParams()
    meta.num_requests, meta.block_size, meta.num_nodes, meta.num_pages = 2, 256, 10, 1
    meta.max_nodes = 2048  # above the 1024-node limit
    assert lib.jt_metadata_build_launch(ctypes.byref(meta), None) == _lib.JT_ERR_INVALID
    assert b"max_nodes" in lib.jt_last_error()
    meta.max_nodes = 64
    assert lib.jt_metadata_build_launch(ctypes.byref(meta), None) == _lib.JT_ERR_INVALID
    assert b"null" in lib.jt_last_error()


def test_workspace_size_geometry(lib):
    size = ctypes.c_size_t(0)
    assert lib.jt_tree_attn_workspace_size(0, 16, 8, 4, 128, ctypes.byref(size)) == _lib.JT_ERR_INVALID
    assert lib.jt_tree_attn_workspace_size(1, 16, 8, 4, 128, None) == _lib.JT_ERR_INVALID
    assert lib.jt_tree_attn_workspace_size(64, 3872, 8, 4, 128, ctypes.byref(size)) == _lib.JT_OK
    small = size.value
    assert small > 0
    assert lib.jt_tree_attn_workspace_size(64, 7744, 8, 4, 128, ctypes.byref(size)) == _lib.JT_OK
    assert size.value >= small


def _params(**overrides):
    p = _lib.JtTreeAttnParams()
    # non-null placeholders: validation rejects geometry before any pointer is used
    for name in ("out", "q", "k_pool", "v_pool", "cu_seqlens_q", "query_to_request",
                 "query_local_row", "prefix_lens", "node_counts", "block_tables", "tree_slots",
                 "qq_bias", "qq_bias_offsets"):
        setattr(p, name, 256)
    p.num_requests, p.total_queries, p.num_kv_heads, p.groups = 1, 16, 1, 4
    p.head_dim, p.block_size, p.table_width = 128, 256, 2
    p.dtype, p.out_dtype = 1, 1
    p.num_blocks = 5
    p.q_stride0, p.q_stride1 = 512, 128
    p.out_stride0, p.out_stride1 = 512, 128
    p.table_stride0 = 2
    p.k_stride0, p.k_stride1, p.k_stride2 = 256 * 128, 128, 128
    p.v_stride0, p.v_stride1, p.v_stride2 = 256 * 128, 128, 128
    p.scale = 128 ** -0.5
    for key, value in overrides.items():
        setattr(p, key, value)
    return p


@pytest.mark.parametrize("field,value,code", [
    ("head_dim", 96, _lib.JT_ERR_UNSUPPORTED),
    ("num_requests", 0, _lib.JT_ERR_INVALID),
    ("groups", 0, _lib.JT_ERR_INVALID),
    ("dtype", 7, _lib.JT_ERR_UNSUPPORTED),
    ("out_dtype", 7, _lib.JT_ERR_INVALID),
    ("q_stride1", 100, _lib.JT_ERR_INVALID),
    ("split_keys", 1000, _lib.JT_ERR_INVALID),
    ("q", None, _lib.JT_ERR_INVALID),
])
def test_launch_validation_precedes_the_device(lib, field, value, code):
    p = _params(**{field: value})
    assert lib.jt_tree_attn_launch(ctypes.byref(p), None) == code
    assert lib.jt_last_error()


def test_status_translation():
    with pytest.raises(ValueError):
        _lib.check(_lib.JT_ERR_INVALID)
    with pytest.raises(ValueError):
        _lib.check(_lib.JT_ERR_UNSUPPORTED)
    with pytest.raises(_lib.KernelLaunchError):
        _lib.check(_lib.JT_ERR_CUDA)
    _lib.check(_lib.JT_OK)


def test_noalloc_rejects_geometry_above_the_static_capacity(lib):
    """A valid launch whose scratch exceeds the 32 MiB static array returns
    JT_ERR_WORKSPACE, naming the capacity, before any CUDA work (no device needed)."""
    p = _params(total_queries=1 << 22, num_kv_heads=8)
    assert lib.jt_tree_attn_launch_noalloc(ctypes.byref(p), None) == _lib.JT_ERR_WORKSPACE
    message = lib.jt_last_error()
    assert b"static capacity" in message and str(32 << 20).encode() in message


def test_commit_slot_limit_without_a_device(lib):
    """Without a visible GPU the per-call commit limit is one CTA's staging (12288
    slots); with one it is that times the SM count."""
    import torch

    limit = lib.jt_kv_commit_max_slots()
    if torch.cuda.is_available():
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        assert limit == 12288 * sms
    else:
        assert limit == 12288
