"""Grouped tensor-core tree attention: the drop-in for the reference's GQA entry point.

``packed_tree_attention_gqa`` keeps the signature, argument meaning and ValueError
behaviour of nanovllm/speculative/jetspec/tree_gqa.py:114-140, but launches the
sm_100a kernels of libjetspec_b200.so through the C ABI instead of Triton.
"""
from __future__ import annotations

import ctypes

import torch

from . import _launch, _lib

SUPPORTED_HEAD_DIMS = (64, 128)
MAX_TREE_NODES = 1024
# jt_tree_attn_workspace_size is a pure function of the launch shape.
_WORKSPACE_SIZES: dict = {}


def _validate(q, k, v, metadata, groups, output_dtype):
    """Operand checks of the reference's shared validator (tree_attention.py:21-37).

    Raises ValueError before any launch and returns the freshly allocated output.
    """
    if q.ndim != 3 or q.shape[0] != metadata.total_queries:
        raise ValueError("packed queries do not match the metadata")
    if k.ndim != 4 or k.shape != v.shape or k.shape[1] != metadata.block_size:
        raise ValueError("packed K/V page geometry does not match metadata")
    if (not q.is_cuda or q.device != k.device or q.device != v.device
            or q.device != metadata.tree_slots.device):
        raise ValueError("packed attention requires CUDA queries, KV and metadata on one device")
    if q.stride(-1) != 1 or k.shape[-1] != q.shape[-1]:
        raise ValueError("unsupported packed query/KV head geometry")
    if (isinstance(groups, bool) or not isinstance(groups, int) or groups <= 0
            or q.shape[1] != k.shape[2] * groups):
        raise ValueError("invalid packed GQA head grouping")
    if q.dtype != k.dtype or k.dtype != v.dtype or q.dtype not in (
            torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("packed Q/K/V must use one supported floating dtype")
    dtype = q.dtype if output_dtype is None else output_dtype
    if dtype not in (q.dtype, torch.float32):
        raise ValueError("output dtype must match input or be FP32 for qualification")
    return torch.empty(q.shape, dtype=dtype, device=q.device)


def _check_metadata(metadata):
    fields = (("cu_seqlens_q", torch.int32), ("query_to_request", torch.int32),
              ("query_local_row", torch.int32), ("prefix_lens", torch.int32),
              ("node_counts", torch.int32), ("block_tables", torch.int32),
              ("tree_slots", torch.int64), ("qq_bias", torch.float32),
              ("qq_bias_offsets", torch.int64))
    for name, dtype in fields:
        tensor = getattr(metadata, name)
        if tensor.dtype != dtype:
            raise ValueError(f"metadata.{name} must be {dtype}")
        if name == "block_tables":
            if tensor.ndim != 2 or tensor.stride(1) != 1:
                raise ValueError("metadata.block_tables must be [requests, width] row-major")
        elif not tensor.is_contiguous():
            raise ValueError(f"metadata.{name} must be contiguous")
    counts = getattr(metadata, "node_counts_host", None)
    if counts and max(counts) > MAX_TREE_NODES:
        raise ValueError(f"trees above {MAX_TREE_NODES} nodes are not supported")


def launch_tree_attention(out, q, k_pool, v_pool, metadata, scale, groups, *,
                          fp32_probability=False, split_keys=0, portable_core=False):
    """Fill ``out`` on the current stream (validated args): directly, or through the
    ``jetspec_b200::tree_attention_`` operator while torch.compile traces the caller."""
    from . import ops

    if ops.compiling():
        torch.ops.jetspec_b200.tree_attention_(
            out, q, k_pool, v_pool, metadata.cu_seqlens_q, metadata.query_to_request,
            metadata.query_local_row, metadata.prefix_lens, metadata.node_counts,
            metadata.block_tables, metadata.tree_slots, metadata.qq_bias,
            metadata.qq_bias_offsets, int(metadata.block_size), float(scale), int(groups),
            bool(fp32_probability), int(split_keys), bool(portable_core))
        return out
    return launch_tree_attention_eager(out, q, k_pool, v_pool, metadata, scale, groups,
                                       fp32_probability=fp32_probability,
                                       split_keys=split_keys, portable_core=portable_core)


def launch_tree_attention_eager(out, q, k_pool, v_pool, metadata, scale, groups, *,
                                fp32_probability=False, split_keys=0, portable_core=False):
    """Fill ``out`` through jt_tree_attn_launch on the current stream (validated args).

    bf16 / f16 operands run on the tensor-core kernels: ``portable_core`` forces the
    warp-level mma.sync core instead of the tcgen05 core (used to cross-check the two
    kernels); head_dim 64 always runs on it.  fp32 operands run on the CUDA-core fp32
    kernel (fp32 products, sums and softmax; no workspace).
    """
    lib = _lib.load_library()
    if q.shape[-1] not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head_dim {q.shape[-1]} is not in {SUPPORTED_HEAD_DIMS}")
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError("tree attention operands must be BF16, FP16 or FP32")
    if k_pool.stride(-1) != 1 or v_pool.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("K/V pools and output need a contiguous head dimension")
    _check_metadata(metadata)
    device = q.device
    num_requests = int(metadata.num_requests)
    total = int(metadata.total_queries)
    kv_heads = int(k_pool.shape[2])
    head_dim = int(q.shape[-1])
    scratch = None
    stream = _launch.raw_stream(device)
    if q.dtype != torch.float32:
        shape = (num_requests, total, kv_heads, int(groups), head_dim)
        nbytes = _WORKSPACE_SIZES.get(shape)
        if nbytes is None:
            size = ctypes.c_size_t(0)
            _lib.check(lib.jt_tree_attn_workspace_size(*shape, ctypes.byref(size)))
            nbytes = _WORKSPACE_SIZES.setdefault(shape, int(size.value))
        scratch = _launch.workspace(device, nbytes, stream)
    p = _lib.JtTreeAttnParams()
    p.out, p.q, p.k_pool, p.v_pool = out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr()
    p.cu_seqlens_q = metadata.cu_seqlens_q.data_ptr()
    p.query_to_request = metadata.query_to_request.data_ptr()
    p.query_local_row = metadata.query_local_row.data_ptr()
    p.prefix_lens = metadata.prefix_lens.data_ptr()
    p.node_counts = metadata.node_counts.data_ptr()
    p.block_tables = metadata.block_tables.data_ptr()
    p.tree_slots = metadata.tree_slots.data_ptr()
    p.qq_bias = metadata.qq_bias.data_ptr()
    p.qq_bias_offsets = metadata.qq_bias_offsets.data_ptr()
    p.num_requests, p.total_queries, p.num_kv_heads = num_requests, total, kv_heads
    p.groups, p.head_dim = int(groups), head_dim
    p.block_size = int(metadata.block_size)
    p.table_width = int(metadata.block_tables.shape[1])
    p.dtype = _launch.DTYPE_CODES[q.dtype]
    p.out_dtype = _launch.DTYPE_CODES[out.dtype]
    p.flags = ((_lib.JT_FLAG_FP32_PROBABILITY if fp32_probability else 0)
               | (_lib.JT_FLAG_PORTABLE_CORE if portable_core else 0))
    p.num_blocks = int(k_pool.shape[0])
    p.q_stride0, p.q_stride1 = q.stride(0), q.stride(1)
    p.out_stride0, p.out_stride1 = out.stride(0), out.stride(1)
    p.table_stride0 = metadata.block_tables.stride(0)
    p.k_stride0, p.k_stride1, p.k_stride2 = k_pool.stride(0), k_pool.stride(1), k_pool.stride(2)
    p.v_stride0, p.v_stride1, p.v_stride2 = v_pool.stride(0), v_pool.stride(1), v_pool.stride(2)
    p.scale = float(scale)
    p.split_keys = int(split_keys)
    p.workspace = None if scratch is None else scratch.data_ptr()
    p.workspace_bytes = 0 if scratch is None else scratch.numel()
    _lib.check(lib.jt_tree_attn_launch(ctypes.byref(p), ctypes.c_void_p(stream)))
    return out


def packed_tree_attention_gqa(q, k_pool, v_pool, metadata, scale, num_queries_per_kv,
                              *, output_dtype=None, query_tile=4, prefix_scalar=True,
                              prune=True, fp32_probability=False):
    """One packed launch of grouped tree attention (bf16/fp16 operands, fp32 softmax).

    ``query_tile``, ``prefix_scalar`` and ``prune`` are the reference's ablation
    switches: they are validated like the reference does and otherwise have no effect
    (the kernel always prunes invisible tree keys and groups all query heads of a KV
    head).  ``fp32_probability`` keeps near-fp32 probabilities in the PV product.
    """
    if query_tile not in (1, 4) or isinstance(query_tile, bool):
        raise ValueError("GQA query tile must be 1 or 4")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("grouped Tensor Core tree attention requires BF16 or FP16")
    if num_queries_per_kv not in (1, 2, 4, 8, 16):
        raise ValueError("grouped tree attention requires power-of-two GQA <=16")
    out = _validate(q, k_pool, v_pool, metadata, num_queries_per_kv, output_dtype)
    return launch_tree_attention(out, q, k_pool, v_pool, metadata, scale, num_queries_per_kv,
                                 fp32_probability=bool(fp32_probability))
