"""Greedy acceptance walk of the verified trees, on the device.

``accept_batch`` keeps the signature and results of the reference's
``accept_batch(logits, trees, offsets, max_depth)``
(nanovllm/speculative/jetspec/serving_ops.py:55-90, called from batch_runtime.py:551-553):
one dict per request with the root-inclusive ``path``, ``accepted_length``,
``correction`` and ``outputs``.  The reference takes the argmax of every node's logits
and walks each tree on the host; here one kernel launch walks all trees with the argmax
taken only for the nodes on the path, and one small download returns the results.
``accept_walk`` is the device-side form: it returns device tensors and never
synchronises, so the accepted path can feed the KV commit without a host round trip.
"""
from __future__ import annotations

import ctypes

import torch

from . import _launch, _lib


def accept_walk(logits: torch.Tensor, token_ids: torch.Tensor, parent_indices: torch.Tensor,
                offsets: torch.Tensor, max_depth: int, *, depths: torch.Tensor | None = None):
    """Walk every packed tree on the device.

    logits [Q, vocab] (bf16/f16/f32, unit stride along the vocabulary), token_ids and
    parent_indices [Q] (int64, parents request-local, -1 for each root), offsets [R + 1]
    (int32 packed node offsets).  Returns (path [R, max_depth + 1] int32,
    accepted_length [R] int32, correction [R] int64, outputs [R, max_depth + 1] int64);
    unused path / output entries are -1.  Launches on the current stream.
    """
    if logits.ndim != 2 or logits.stride(-1) != 1:
        raise ValueError("logits must be [nodes, vocab] with a contiguous vocabulary axis")
    if logits.dtype not in _launch.DTYPE_CODES:
        raise ValueError("logits must be bf16, f16 or f32")
    nodes = logits.shape[0]
    if token_ids.shape != (nodes,) or parent_indices.shape != (nodes,):
        raise ValueError("token_ids and parent_indices must hold one entry per logits row")
    if offsets.ndim != 1 or offsets.numel() < 2:
        raise ValueError("offsets must be [requests + 1]")
    if max_depth < 0:
        raise ValueError("max_depth must be non-negative")
    device = logits.device
    tensors = [token_ids, parent_indices, offsets] + ([depths] if depths is not None else [])
    if not logits.is_cuda or any(t.device != device for t in tensors):
        raise ValueError("acceptance walk requires CUDA tensors on one device")
    token_ids = token_ids.to(torch.int64).contiguous()
    parent_indices = parent_indices.to(torch.int64).contiguous()
    offsets = offsets.to(torch.int32).contiguous()
    if depths is not None:
        depths = depths.to(torch.int64).contiguous()
    requests = offsets.numel() - 1
    width = max_depth + 1
    path = torch.empty((requests, width), dtype=torch.int32, device=device)
    accepted = torch.empty(requests, dtype=torch.int32, device=device)
    correction = torch.empty(requests, dtype=torch.int64, device=device)
    outputs = torch.empty((requests, width), dtype=torch.int64, device=device)
    p = _lib.JtAcceptWalkParams()
    p.logits = logits.data_ptr()
    p.token_ids, p.parent_indices = token_ids.data_ptr(), parent_indices.data_ptr()
    p.depths = depths.data_ptr() if depths is not None else None
    p.offsets = offsets.data_ptr()
    p.path, p.accepted_length = path.data_ptr(), accepted.data_ptr()
    p.correction, p.outputs = correction.data_ptr(), outputs.data_ptr()
    p.logits_stride0 = logits.stride(0)
    p.logits_dtype = _launch.DTYPE_CODES[logits.dtype]
    p.vocab, p.num_requests = logits.shape[1], requests
    p.max_depth, p.path_stride = int(max_depth), width
    p.num_nodes = nodes
    lib = _lib.load_library()
    _lib.check(lib.jt_accept_walk_launch(ctypes.byref(p), _launch.stream_handle(device)))
    return path, accepted, correction, outputs


def _host_list(tree, host_name, name):
    values = getattr(tree, host_name, None)
    return values if values is not None else getattr(tree, name).tolist()


def _packed(tensors, device):
    """One flat device tensor of the trees' per-node values.  build_trees leaves them as
    back-to-back views of one packed allocation; then that storage is used as it is,
    otherwise the pieces are concatenated."""
    first = tensors[0]
    start, total = first.storage_offset(), 0
    contiguous = all(
        t.device == device and t.dtype == first.dtype and t.dim() == 1 and
        (t.numel() <= 1 or t.stride(0) == 1) and
        t.untyped_storage().data_ptr() == first.untyped_storage().data_ptr() and
        t.storage_offset() == start + (total := total + t.numel()) - t.numel()
        for t in tensors)
    if contiguous:
        return first.as_strided((total,), (1,), start)
    return torch.cat([t.reshape(-1).to(device) for t in tensors])


def accept_batch(logits, trees, offsets, max_depth):
    """The reference's accept_batch results, walked on the device (one launch, one download).

    ``trees`` carry ``token_ids``, ``parent_indices`` and ``depth`` (device tensors, as
    build_trees leaves them) and ``num_nodes``; ``offsets`` are the packed node offsets
    (metadata.query_offsets).  Raises RuntimeError when the depths along a path are not
    0, 1, 2, ... (the reference's check).
    """
    device = logits.device
    offsets = [int(o) for o in offsets]
    if (len(offsets) != len(trees) + 1 or offsets[0] != 0 or offsets[-1] != logits.shape[0] or
            any(b - a != int(t.num_nodes) for a, b, t in zip(offsets, offsets[1:], trees))):
        raise ValueError("offsets must be the packed node offsets of the trees")
    token_ids = _packed([t.token_ids for t in trees], device)
    parents = _packed([t.parent_indices for t in trees], device)
    offs = torch.tensor(offsets, dtype=torch.int32, device=device)
    path, accepted, correction, outputs = accept_walk(logits, token_ids, parents, offs,
                                                      max_depth)
    rows = torch.cat((path.to(torch.int64), accepted.to(torch.int64)[:, None],
                      correction[:, None], outputs), dim=1).tolist()  # the one download
    width = max_depth + 1
    results = []
    for tree, row in zip(trees, rows):
        length = row[width] + 1
        node_path = row[:length]
        depths = _host_list(tree, "host_depths", "depth")
        if any(depths[node] != i for i, node in enumerate(node_path)):
            raise RuntimeError("accepted RoPE positions do not match canonical tail")
        results.append({"path": node_path, "accepted_length": length - 1,
                        "correction": row[width + 1],
                        "outputs": row[width + 2:width + 2 + length]})
    return results
