"""Tree-node KV write into scratch slots before verification.

``scatter_tree_kv`` is the non-fused node write of the verifier
(nanovllm/models/qwen3.py:255-258: ``k_pool[slot // bs, slot % bs] = k`` and the same
for V) as one launch of the warp-per-token store kernel.  ``rope_scatter`` /
``rope_scatter_prevalidated`` are the fused HF-order RoPE + scatter of
nanovllm/speculative/jetspec/tree_fusion.py (same signatures, checks and messages), as
one launch of the sm_100a rope_scatter kernel, bit-exact with eager PyTorch RoPE.
"""
from __future__ import annotations

import torch

from .attention import _store


def scatter_tree_kv(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                    v_pool: torch.Tensor, node_slots: torch.Tensor) -> None:
    """Write node K/V rows [Q, kv_heads, dim] to their scratch slots (bit-exact)."""
    if k.ndim != 3 or v.shape != k.shape or node_slots.shape != (k.shape[0],):
        raise ValueError("node K/V must be [rows, kv_heads, dim] with one slot per row")
    from . import ops

    if ops.compiling():
        torch.ops.jetspec_b200.kv_store_(k, v, k_pool, v_pool, node_slots.contiguous())
        return
    _store(k, v, k_pool, v_pool, node_slots.contiguous())


# ---- fused HF-order RoPE + node K/V scatter (tree_fusion.py:181-199) -------------------
def _memory_range(tensor):
    start = tensor.data_ptr()
    span = 1 + sum((size - 1) * stride for size, stride in zip(tensor.shape, tensor.stride()))
    return start, start + span * tensor.element_size()


def _overlap(a, b):
    a0, a1 = _memory_range(a)
    b0, b1 = _memory_range(b)
    return a0 < b1 and b0 < a1


def _injective(tensor):
    """Host-only check that no two indices of a strided view share an address."""
    span = 1
    for stride, size in sorted((stride, size) for stride, size in
                               zip(tensor.stride(), tensor.shape) if size > 1):
        if stride < span:
            return False
        span += (size - 1) * stride
    return True


def _validate_rope(q, k, v, positions, cache, k_pool, v_pool, node_slots, out):
    """The reference's rope_scatter checks (tree_fusion.py:107-169), same messages."""
    tensors = (q, k, v, positions, cache, k_pool, v_pool, node_slots)
    if q.ndim != 3 or k.ndim != 3 or v.shape != k.shape:
        raise ValueError("Q/K/V must be [rows,heads,dim] with equal K/V geometry")
    rows, q_heads, dim = q.shape
    if (rows < 1 or q_heads < 1 or k.shape[0] != rows or k.shape[1] < 1 or
            k.shape[2] != dim or dim < 2 or dim % 2 or dim > 256 or q_heads % k.shape[1]):
        raise ValueError("invalid nonempty Q/K/V GQA or even head geometry")
    if q.dtype not in (torch.bfloat16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("RoPE fusion supports matching BF16 or FP32 Q/K/V")
    if (positions.shape != (rows,) or node_slots.shape != (rows,) or
            positions.dtype not in (torch.int32, torch.int64) or
            node_slots.dtype not in (torch.int32, torch.int64)):
        raise ValueError("positions and node_slots must be integer [rows] vectors")
    if (cache.ndim not in (2, 3) or cache.shape[-1] != dim or cache.shape[0] < 1 or
            (cache.ndim == 3 and cache.shape[1] != 1) or
            cache.dtype not in (torch.bfloat16, torch.float32)):
        raise ValueError("cos/sin cache must be BF16/FP32 [positions,dim] or [positions,1,dim]")
    if (k_pool.ndim != 4 or v_pool.shape != k_pool.shape or k_pool.shape[0] < 1 or
            k_pool.shape[1] < 1 or tuple(k_pool.shape[2:]) != (k.shape[1], dim) or
            k_pool.dtype != q.dtype or v_pool.dtype != q.dtype):
        raise ValueError("KV pools must match [pages,page_size,kv_heads,dim] and Q/K/V dtype")
    if any(any(stride <= 0 for stride in t.stride()) for t in tensors):
        raise ValueError("RoPE fusion requires positive tensor strides")
    if not q.is_cuda or any(t.device != q.device for t in tensors):
        raise ValueError("RoPE fusion requires CUDA tensors on one device")
    if not _injective(k_pool) or not _injective(v_pool):
        raise ValueError("KV pool layouts must not have overlapping write addresses")
    if out is not None:
        if (out.shape != q.shape or out.dtype != q.dtype or out.device != q.device or
                any(stride <= 0 for stride in out.stride())):
            raise ValueError("output must match Q shape, dtype and device with positive strides")
        if not _injective(out):
            raise ValueError("output layout must not have overlapping write addresses")
        if any(_overlap(out, t) for t in tensors):
            raise ValueError("output must not alias any source or KV pool")
    if _overlap(k_pool, v_pool):
        raise ValueError("K and V pool views must not overlap")
    sources = (q, k, v, positions, cache, node_slots)
    if any(_overlap(pool, source) for pool in (k_pool, v_pool) for source in sources):
        raise ValueError("KV pools must not overlap source tensors")
    # The external boundary checks device VALUES and therefore synchronises; the
    # prevalidated serving entry below never does.
    if bool(((positions < 0) | (positions >= cache.shape[0])).any().item()):
        raise ValueError("RoPE positions lie outside the cos/sin cache")
    capacity = k_pool.shape[0] * k_pool.shape[1]
    if bool(((node_slots < 0) | (node_slots >= capacity)).any().item()):
        raise ValueError("node slots lie outside the KV pool")
    if node_slots.unique().numel() != rows:
        raise ValueError("node slots must be unique to avoid KV write races")


def rope_scatter(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots, *, out=None):
    """Validate, return HF-order rotated Q and scatter rotated K / raw V in place.

    Drop-in for rope_scatter (nanovllm/speculative/jetspec/tree_fusion.py:172-178):
    cache rows hold ``[cos_half | sin_half]``; slots must be in range and unique.
    """
    _validate_rope(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots, out)
    if out is None:
        out = torch.empty_like(q)
    return rope_scatter_prevalidated(q, k, v, positions, cos_sin_cache, k_pool, v_pool,
                                     node_slots, out)


_DT = {torch.bfloat16: 0, torch.float32: 2}


def rope_scatter_prevalidated(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots, out):
    """Launch-only serving boundary (tree_fusion.py:181-199): one sm_100a kernel, no
    allocation, download or synchronisation; the caller guarantees the invariants that
    ``rope_scatter`` checks."""
    from . import ops

    if ops.compiling():
        torch.ops.jetspec_b200.rope_scatter_(q, k, v, positions, cos_sin_cache, k_pool, v_pool,
                                             node_slots, out)
        return out
    return _rope_scatter_launch(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots,
                                out)


def _rope_scatter_launch(q, k, v, positions, cos_sin_cache, k_pool, v_pool, node_slots, out):
    """jt_rope_scatter_launch on the current stream."""
    import ctypes

    from . import _launch, _lib

    lib = _lib.load_library()
    p = _lib.JtRopeScatterParams()
    p.q, p.k, p.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.positions, p.cos_sin_cache = positions.data_ptr(), cos_sin_cache.data_ptr()
    p.node_slots, p.out = node_slots.data_ptr(), out.data_ptr()
    p.k_pool, p.v_pool = k_pool.data_ptr(), v_pool.data_ptr()
    p.dtype = _DT[q.dtype]
    p.cache_dtype = _DT[cos_sin_cache.dtype]
    p.positions_is_int64 = int(positions.dtype == torch.int64)
    p.slots_is_int64 = int(node_slots.dtype == torch.int64)
    p.rows, p.q_heads, p.head_dim = q.shape
    p.kv_heads = k.shape[1]
    p.page_size, p.num_pages = k_pool.shape[1], k_pool.shape[0]
    p.q_stride0, p.q_stride1, p.q_stride2 = q.stride()
    p.k_stride0, p.k_stride1, p.k_stride2 = k.stride()
    p.v_stride0, p.v_stride1, p.v_stride2 = v.stride()
    p.positions_stride, p.slots_stride = positions.stride(0), node_slots.stride(0)
    p.cache_stride0, p.cache_stride_last = cos_sin_cache.stride(0), cos_sin_cache.stride(-1)
    p.out_stride0, p.out_stride1, p.out_stride2 = out.stride()
    p.kp_stride0, p.kp_stride1, p.kp_stride2, p.kp_stride3 = k_pool.stride()
    p.vp_stride0, p.vp_stride1, p.vp_stride2, p.vp_stride3 = v_pool.stride()
    _lib.check(lib.jt_rope_scatter_launch(ctypes.byref(p), _launch.stream_handle(q.device)))
    return out
